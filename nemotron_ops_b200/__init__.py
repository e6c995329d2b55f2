"""nemotron_ops_b200: B200 (sm_100a) weight-streaming decode ops of the nemotron_ops ``bolt`` domain.

The compute lives in libbolt_b200.so (hand-written CUDA for sm_100a behind the C ABI of
include/bolt_b200.h).  ``nemotron_ops_b200.ops`` exposes the ops on torch CUDA tensors with the
reference's op names; ``nemotron_ops_b200.sharded`` runs MoeVerify with experts sharded across
the ranks of a torch.distributed process group.
"""
from ._lib import LIB_PATH, lib  # noqa: F401

__all__ = ["LIB_PATH", "lib"]
