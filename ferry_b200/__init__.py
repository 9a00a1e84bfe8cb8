"""ferry_b200 -- B200-native sparse KV-cache miss-stream decode path.

The hot path (top-k page selection, miss detection against the HBM page cache,
miss gather from pinned host memory, paged sparse decode attention) is
hand-written CUDA for sm_100a in ``csrc/``, exported through the C ABI in
``include/ferry_cuda.h`` as ``libferry_cuda.so``. This package is the host side:
``_abi`` binds the library, ``engine`` drives it, ``workload`` generates the
seeded synthetic inputs.
"""
from ._abi import FerryError, lib  # noqa: F401
from .workload import CFG1, WORKLOADS, Schedule, Workload, q_stream, small  # noqa: F401

__version__ = "0.1.0"
