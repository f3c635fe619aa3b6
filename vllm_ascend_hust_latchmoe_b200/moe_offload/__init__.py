"""Offload runtime of the slot-bank MoE layer: slot bank, pinned host store, transfer engine,
wave planning and the runtime that owns them (mirrors ``vllm_moe_offload_ascend.moe_offload``)."""
