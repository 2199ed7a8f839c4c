"""Process groups, NCCL baseline collectives and the fused NVLink collectives."""
from . import comm, state  # noqa: F401
