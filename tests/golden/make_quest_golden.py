"""Regenerate quest_selector.npz: page sets chosen by the reference's own Quest
selector, Selector.on_layer(method="quest") of tools/capture_miss_trace.py
(lines 128-159, run here on CPU torch), for keys taken from this repository's
procedural KV pool and seeded fp16 queries.

    python tests/golden/make_quest_golden.py [--ref <reference checkout>]

The reference checkout defaults to a folder named ``reference`` beside this
repository's checkout. Runs only where that checkout, torch and transformers
are present; the tests read the fixture it writes.

Keys: pool units of ``oracle.kv_gen(seed, ...)`` (bit-identical to
``ferry_kv_generate``) in the layout the decode path uses -- request r, layer
l, kv head h, page p is unit ((r * L + l) * Hkv + h) * N + p, K in its first
4 KiB. A context of T tokens covers pages 0 .. T // 16 - 1 (the selector
drops a ragged tail; T % 16 tokens of the next page are passed to it and
ignored). Queries: fp16 values of a seeded normal draw, redrawn until the
float64 Quest scores separate the k-th and (k+1)-th page by a margin of 1e-3
of the largest score (so fp32 summation-order differences cannot change the
set).
"""
import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

# name: requests, layers, q heads, kv heads, pages per lane (N), context tokens, top-k
CASES = {
    "cfg1_shape": (1, 1, 32, 32, 256, 4096, 64),
    "gqa8": (2, 2, 64, 8, 512, 8192, 128),
    "ragged": (1, 1, 8, 2, 64, 1000, 16),
    "few_pages": (1, 1, 4, 4, 16, 200, 16),
}
KV_SEED = 4242


def quest_scores64(q, keys, page_tokens=16):
    """float64 Quest scores (for the margin check only)."""
    Hq, Hkv = q.shape[0], keys.shape[0]
    n_pages = keys.shape[1] // page_tokens
    kp = keys[:, : n_pages * page_tokens].astype(np.float64).reshape(Hkv, n_pages, page_tokens, -1)
    kmin, kmax = kp.min(2), kp.max(2)
    qq = q.astype(np.float64).reshape(Hkv, Hq // Hkv, 1, -1)
    b = np.maximum(qq * kmax[:, None], qq * kmin[:, None]).sum(-1)  # Hkv, G, pages
    return b.max(1).max(0)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.path.join(os.path.dirname(ROOT), "reference"))
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.ref, "tools"))
    import torch
    from capture_miss_trace import Selector

    oracle.build()
    out = {"kv_seed": np.int64(KV_SEED)}
    for name, (R, L, Hq, Hkv, N, T, k) in CASES.items():
        units = oracle.kv_gen(KV_SEED, 0, R * L * Hkv * N)
        K = units.reshape(R, L, Hkv, N, 2, 16, 128)[:, :, :, :, 0].view(np.float16)  # R L Hkv N 16 128
        sel = np.full((R, L, k), -1, np.int64)
        qbits = np.zeros((R, L, Hq, 128), np.uint16)
        rng = np.random.default_rng([KV_SEED, R, L, Hq, Hkv, N, T, k])
        for r in range(R):
            for li in range(L):
                keys = K[r, li].reshape(Hkv, N * 16, 128)[:, :T]
                n_pages = T // 16
                while True:
                    q = rng.standard_normal((Hq, 128)).astype(np.float16)
                    if n_pages <= k:
                        break
                    sc = np.sort(quest_scores64(q, keys))[::-1]
                    if sc[k - 1] - sc[k] > 1e-3 * np.abs(sc).max():
                        break
                s = Selector("quest", page_tokens=16, block_tokens=4, sel_pages=k, num_layers=L,
                             num_heads=Hq, num_kv_heads=Hkv, head_dim=128, scaling=128 ** -0.5)
                s.on_layer(li, torch.from_numpy(q).view(1, Hq, 1, 128),
                           torch.from_numpy(np.ascontiguousarray(keys)).view(1, Hkv, T, 128))
                pages = s.step_pages()[li]
                sel[r, li, : len(pages)] = pages
                qbits[r, li] = q.view(np.uint16)
        out[f"{name}_shape"] = np.array([R, L, Hq, Hkv, N, T, k], np.int64)
        out[f"{name}_q"] = qbits
        out[f"{name}_sel"] = sel
    np.savez_compressed(os.path.join(HERE, "quest_selector.npz"), **out)
    print("wrote quest_selector.npz:", {n: CASES[n] for n in CASES})


if __name__ == "__main__":
    main()
