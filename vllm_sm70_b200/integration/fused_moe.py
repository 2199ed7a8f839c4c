"""Fused-MoE area: routing (U3 provider in ``models/router.py``) and the
grouped expert GEMMs (``ops/moe.py``)."""


def register() -> None:
    return None
