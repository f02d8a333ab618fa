"""Generates the golden fixtures in this directory from the reference's own code.

  quant_*.npz  the reference's unmodified host quantizer (src/quant_format.cuh,
               built by oracle/build_oracle.py into oracle/_ref/ref_quant) on
               seeded and edge-value FP16 matrices: inputs and its packed codes,
               scales and zero-points.          (CPU: python tests/golden/make_golden.py)
  gemv_*.npz   the reference's own GPU kernels (src/{split,int4,reference}_gemv.cu
               and scan_outliers_block, built for sm_100a into
               oracle/_ref/libdqref_gpu.so) on seeded inputs: W, x, k, the three
               GEMV outputs and the detector's list/count/statistics.
               The reference's split kernel stages packed bytes for rows 0..1 of
               each 4-row block only (src/split_gemv.cu:85-93), so its output is
               kept for rows with row % 4 in {0, 1}; `split_rows` marks them.
                                                (B200: python tests/golden/make_golden.py --gpu OUTDIR)
Fixture inputs come from seeded numpy generators; nothing is written from memory.
"""
from __future__ import annotations

import argparse
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, os.path.join(ROOT, "dyn-quant_b200")]

import oracle as O  # noqa: E402
from dyn_quant import synth  # noqa: E402


def quant_inputs():
    edge = np.zeros((8, 256), np.float16)
    edge[1, :] = 1.5
    edge[2, ::2] = -0.0
    edge[3, 5] = np.inf
    edge[4, 7] = -np.inf
    edge[5, 9] = np.nan
    edge[6, :128] = np.nan
    edge[7, 3] = 65504
    edge[7, 4] = -65504
    edge[0, 130:140] = np.float16(6e-8)
    rng = np.random.default_rng(11)
    wide = (rng.standard_normal((16, 512)) * np.array([1e-4, 1.0, 300.0, 2e4])[rng.integers(0, 4, (16, 1))])
    return {
        "edge_8x256": edge,
        "normal_64x512": synth.weights(64, 512, seed=7),
        "normal_33x1024": synth.weights(33, 1024, seed=8),
        "wide_16x512": np.clip(wide, -65504, 65504).astype(np.float16),
    }


def gemv_inputs():
    return {
        "normal_256x1024_f2": (synth.weights(256, 1024, seed=21), synth.activation(1024, 0.02, seed=22), 3.0),
        "normal_128x4096_f1": (synth.weights(128, 4096, seed=23), synth.activation(4096, 0.01, seed=24), 3.0),
        "t3_64x2048_k2": (synth.weights(64, 2048, seed=25), synth.activation(2048, 0.0, seed=26, dist="t3"), 2.0),
    }


def make_quant(outdir):
    if not O.ref_quant_available():
        raise SystemExit("oracle/_ref/ref_quant missing: run python oracle/build_oracle.py first")
    for name, w in quant_inputs().items():
        p, s, z = O.ref_quantize(w)
        np.savez_compressed(os.path.join(outdir, f"quant_{name}.npz"), w=w.view(np.uint16), packed=p,
                            scales=s.view(np.uint16), zeros=z.view(np.uint16))
        print("wrote", name)


def make_gemv(outdir):
    import torch
    L = C.CDLL(O.REF_GPU_LIB)
    vp = C.c_void_p
    L.dqref_split_gemv.argtypes = [vp, vp, vp, vp, vp, vp, C.c_int, C.c_int, C.c_float, vp]
    L.dqref_int4_gemv.argtypes = [vp, vp, vp, vp, vp, C.c_int, C.c_int, vp]
    L.dqref_reference_gemv.argtypes = [vp, vp, vp, C.c_int, C.c_int, vp]
    L.dqref_detect.argtypes = [vp, C.c_int, C.c_float, vp, vp, vp, vp]
    dev = torch.device("cuda", 0)
    for name, (w, x, k) in gemv_inputs().items():
        d_out, d_in = w.shape
        p, s, z = O.ref_quantize(w)
        t = {n: torch.from_numpy(np.ascontiguousarray(a)).to(dev) for n, a in
             (("p", p), ("s", s), ("z", z), ("w", w), ("x", x))}
        ys = {n: torch.zeros(d_out, dtype=torch.float16, device=dev) for n in ("split", "int4", "ref")}
        idx = torch.zeros(d_in // 4, dtype=torch.int32, device=dev)
        cnt = torch.zeros(1, dtype=torch.int32, device=dev)
        st = torch.zeros(4, dtype=torch.float32, device=dev)
        P = lambda a: C.c_void_p(a.data_ptr())  # noqa: E731
        assert L.dqref_split_gemv(P(t["p"]), P(t["s"]), P(t["z"]), P(t["w"]), P(t["x"]), P(ys["split"]),
                                  d_out, d_in, k, None) == 0
        assert L.dqref_int4_gemv(P(t["p"]), P(t["s"]), P(t["z"]), P(t["x"]), P(ys["int4"]), d_out, d_in,
                                 None) == 0
        assert L.dqref_reference_gemv(P(t["w"]), P(t["x"]), P(ys["ref"]), d_out, d_in, None) == 0
        assert L.dqref_detect(P(t["x"]), d_in, k, P(idx), P(cnt), P(st), None) == 0
        torch.cuda.synchronize()
        n = int(cnt.item())
        np.savez_compressed(
            os.path.join(outdir, f"gemv_{name}.npz"), w=w.view(np.uint16), x=x.view(np.uint16), k=np.float32(k),
            y_split=ys["split"].cpu().numpy().view(np.uint16), split_rows=(np.arange(d_out) % 4) < 2,
            y_int4=ys["int4"].cpu().numpy().view(np.uint16), y_ref=ys["ref"].cpu().numpy().view(np.uint16),
            indices=idx.cpu().numpy()[:n], stats=st.cpu().numpy())
        print("wrote", name, "outliers", n)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpu", metavar="OUTDIR", help="run the reference's GPU kernels and write gemv_*.npz there")
    args = ap.parse_args()
    if args.gpu:
        os.makedirs(args.gpu, exist_ok=True)
        make_gemv(args.gpu)
    else:
        make_quant(HERE)


if __name__ == "__main__":
    main()
