"""Generates the golden fixtures in this folder (run in the build container, where
the reference sources are present):

  bilinear_ref.npz -- outputs of the reference's OWN host bilinear reference
                      (cpu_bilinear_upsample_reference, benchmarks/upsample_benchmark.cu:24-108),
                      compiled from its source by oracle/Makefile into oracle/_ref/, on seeded
                      U(-1, 1) inputs (the reference benchmark's distribution, :253-272).
  neck_small.npz   -- digests of the fp32 CPU neck oracle on a small seeded problem
                      (per level: sum, sum of squares and 2048 sampled values).

    make -C oracle REF=<reference checkout> && python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import fpn_oracle as O  # noqa: E402

# (N, C, ih, iw, oh, ow, align_corners)
BILINEAR_CASES = [
    (1, 3, 5, 7, 10, 14, 0),        # exact 2x
    (2, 4, 25, 42, 50, 84, 0),      # Swin 1333x800 top level (2x)
    (1, 2, 50, 84, 100, 167, 0),    # non-2x: 84 -> 167
    (1, 1, 84, 50, 167, 100, 0),    # non-2x along H
    (1, 3, 6, 9, 11, 17, 1),        # align_corners
    (1, 1, 1, 1, 3, 3, 0),          # single pixel
    (1, 2, 4, 4, 1, 1, 0),          # output of one pixel
    (1, 2, 9, 9, 4, 4, 0),          # downsample
    (1, 2, 13, 19, 25, 38, 0),      # R50 P6 <- P5 sizes reversed (odd)
]


def reference_bilinear(lib, x, oh, ow, ac):
    n, c, ih, iw = x.shape
    out = np.zeros((n, c, oh, ow), np.float32)
    lib.ref_cpu_bilinear_upsample_f32(x.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p),
                                      n, c, ih, iw, oh, ow, ac)
    return out


def main():
    lib = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libref_bilinear.so"))
    lib.ref_cpu_bilinear_upsample_f32.restype = None
    lib.ref_cpu_bilinear_upsample_f32.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 7
    rs = np.random.RandomState(42)
    arrays = {}
    for i, (n, c, ih, iw, oh, ow, ac) in enumerate(BILINEAR_CASES):
        x = rs.uniform(-1, 1, (n, c, ih, iw)).astype(np.float32)
        arrays[f"case{i}_shape"] = np.array([n, c, ih, iw, oh, ow, ac], np.int64)
        arrays[f"case{i}_in"] = x
        arrays[f"case{i}_out"] = reference_bilinear(lib, x, oh, ow, ac)
    np.savez_compressed(HERE / "bilinear_ref.npz", **arrays)

    # small neck: R50-like channel ratios, odd top-down sizes (3x4 -> 5x7 -> 10x14 -> 20x28)
    chans = (64, 128, 128, 256)
    sizes = [(20, 28), (10, 14), (5, 7), (3, 4)]
    feats = O.make_features(1, chans, sizes, seed=7, dist="normal")
    wts = O.make_weights(chans, seed=8, bias_scale=0.1)
    outs = O.fpn_neck(feats, wts)
    g = np.random.RandomState(3)
    neck = {"chans": np.array(chans), "sizes": np.array(sizes)}
    for k, o in enumerate(outs):
        a = o.numpy().astype(np.float64)
        idx = g.randint(0, a.size, 2048)
        neck[f"P{k + 2}_shape"] = np.array(a.shape)
        neck[f"P{k + 2}_sum"] = a.sum()
        neck[f"P{k + 2}_sumsq"] = (a * a).sum()
        neck[f"P{k + 2}_idx"] = idx
        neck[f"P{k + 2}_val"] = a.reshape(-1)[idx].astype(np.float32)
    np.savez_compressed(HERE / "neck_small.npz", **neck)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    torch.manual_seed(0)
    main()
