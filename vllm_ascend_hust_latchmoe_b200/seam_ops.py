"""Seam custom ops (placeholder until the op layer lands)."""


def register_ops() -> None:
    return None
