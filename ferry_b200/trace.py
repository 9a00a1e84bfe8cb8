"""FMT1 real-selection traces: write (for tools and tests) and load (through
the library's ``ferry_trace_load``).

Format (the reference's capture tool, tools/capture_miss_trace.py:316-317,
368-370): header ``<4sIIIIIIIII`` = b"FMT1", version 1, requests, steps,
layers, page_tokens, block_tokens, kv_heads, head_dim, sel_pages; then per
(request, step, layer) a little-endian u16 count and that many u32 block ids.
"""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np

from . import _abi


def write_fmt1(path: str, ids: np.ndarray, page_tokens: int = 16, block_tokens: int = 4,
               kv_heads: int = 8, head_dim: int = 128, counts: np.ndarray | None = None,
               header_override: dict | None = None) -> None:
    """ids: [requests][steps][layers][sel_blocks] uint32 raw block ids."""
    R, S, L, G = ids.shape
    hdr = dict(version=1, requests=R, steps=S, layers=L, page_tokens=page_tokens,
               block_tokens=block_tokens, kv_heads=kv_heads, head_dim=head_dim,
               sel_pages=G // (page_tokens // block_tokens))
    hdr.update(header_override or {})
    with open(path, "wb") as f:
        f.write(struct.pack("<4sIIIIIIIII", b"FMT1", hdr["version"], hdr["requests"], hdr["steps"],
                            hdr["layers"], hdr["page_tokens"], hdr["block_tokens"], hdr["kv_heads"],
                            hdr["head_dim"], hdr["sel_pages"]))
        for r in range(R):
            for s in range(S):
                for l in range(L):
                    n = G if counts is None else int(counts[r, s, l])
                    f.write(struct.pack("<H", n))
                    f.write(np.ascontiguousarray(ids[r, s, l, :n], "<u4").tobytes())


def load(path: str, requests: int, steps: int, layers: int, sel_blocks: int, kv_heads: int = 8,
         head_dim: int = 128):
    """Dense block ids [requests][steps][layers][sel_blocks] (first-seen
    order), distinct-id count, slab capacity. Raises FerryError on mismatch."""
    n = requests * steps * layers * sel_blocks
    out = np.zeros(n, np.int64)
    uniq = C.c_int64()
    slab = C.c_int32()
    _abi.call("ferry_trace_load", path.encode(), requests, steps, layers, sel_blocks, kv_heads, head_dim,
              out.ctypes.data_as(C.c_void_p), C.c_int64(n), C.byref(uniq), C.byref(slab))
    return out.reshape(requests, steps, layers, sel_blocks), int(uniq.value), int(slab.value)


def synthetic_ids(requests: int, steps: int, layers: int, sel_blocks: int, seed: int = 0,
                  group: int = 4, reuse: float = 0.7) -> np.ndarray:
    """Raw u32 ids shaped like real captures: requests in prefix groups share
    ids, each step re-selects ~reuse of the previous step's blocks."""
    rng = np.random.default_rng(seed)
    out = np.zeros((requests, steps, layers, sel_blocks), np.uint32)
    for r in range(requests):
        base = rng.integers(1, 2**32 - 1, size=4 * sel_blocks, dtype=np.uint64).astype(np.uint32)
        shared = np.random.default_rng([seed, r // group]).integers(1, 2**32 - 1, size=2 * sel_blocks,
                                                                     dtype=np.uint64).astype(np.uint32)
        pool = np.concatenate([base, shared])
        for l in range(layers):
            prev = rng.choice(pool, sel_blocks)
            for s in range(steps):
                keep = rng.random(sel_blocks) < reuse
                cur = np.where(keep, rng.choice(prev, sel_blocks), rng.choice(pool, sel_blocks))
                out[r, s, l] = cur
                prev = cur
    return out
