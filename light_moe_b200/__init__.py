"""light_moe_b200 -- the MoE-layer hot path of light-moe, rebuilt for B200 (sm_100a).

* ``capi``   ctypes view of the C ABI in ``include/lmoe_b200.h`` (``lib/liblmoe_b200.so``)
* ``ops``    the reference's ``light_moe._C`` operator surface plus the W4A16 / layer ops
* ``layer``  ``W4A16Experts`` and ``W4A16MoELayer`` (drop-in for ``SparseMoEBlock``)
* ``expert_parallel``  the expert-parallel layer over NCCL

Build with ``python -m light_moe_b200.build``.  Nothing here falls back to a CPU or
PyTorch implementation: an op called without the built library raises.
"""
__version__ = "0.1.0"

from . import capi, ops  # noqa: F401
