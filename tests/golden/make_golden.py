"""Generate the golden vectors in tests/golden/*.npz from the REFERENCE itself.

Run where a checkout of the reference exists (--reference names it; the default is the build
container's checkout):

    python tests/golden/make_golden.py [--reference PATH]

For every case it records what the reference produces:
  qweight, scales, zeros   int4gemv/quant.py:14-29 (quantize) on seeded float32 weights w
  deq                      int4gemv/quant.py:47-53 (dequantize), small cases only
  y_ref                    int4gemv/reference.py:8-10 (torch fp32 dequantise-then-matmul)
  y_seq                    csrc/sequential.cpp:11-54, the reference's compiled CPU path
                           (oracle/_ref, built by oracle/build_ref.py)
  pack_wrap.npz            int4gemv/quant.py:32-37 (pack) on int32 values inside and outside 0..15
The tests then pin the C oracle (oracle/w4a16_oracle.c) to these, and the CUDA kernels to both.
Nothing on the GPU box reads the reference: only these .npz files travel.
"""

from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]

# (name, M, N, K, group_size, keep_w): shapes chosen to cover M tiles (1, 3, 5, 8, 16), ragged N,
# every legal kind of group size (8-multiple, 32-multiple, 128) and K that is / is not a multiple
# of 1024.
CASES = [
    ("m1_n64_k256_g128", 1, 64, 256, 128, True),
    ("m3_n37_k384_g128", 3, 37, 384, 128, True),
    ("m8_n128_k1024_g64", 8, 128, 1024, 64, False),
    ("m2_n20_k64_g16", 2, 20, 64, 16, True),
    ("m2_n24_k96_g8", 2, 24, 96, 8, True),
    ("m5_n48_k512_g32", 5, 48, 512, 32, True),
    ("m16_n32_k512_g128", 16, 32, 512, 128, True),
    ("m32_n40_k256_g128", 32, 40, 256, 128, True),
    ("m1_n96_k2048_g128", 1, 96, 2048, 128, False),
    ("m4_n150_k3072_g128", 4, 150, 3072, 128, False),
]


def edge_weights() -> np.ndarray:
    """Rows that hit the corners of quantize: all zero (scale clamped to 1e-6), all positive
    (zero point 0), all negative (zero point 15), constant, tiny, large, ties, random."""
    k = 256
    rng = np.random.default_rng(7)
    rows = [
        np.zeros(k),
        np.abs(rng.standard_normal(k)) * 0.02 + 0.001,
        -np.abs(rng.standard_normal(k)) * 0.02 - 0.001,
        np.full(k, 0.5),
        rng.standard_normal(k) * 1e-8,
        rng.standard_normal(k) * 100.0,
        np.linspace(-1.0, 1.0, k),
        # multiples of 1/30 over [-0.5, 0.5]: w / s lands on .5 ties for several entries
        np.round(rng.uniform(-15, 15, k)) / 30.0,
        rng.standard_normal(k) * 0.02,
    ]
    return np.stack(rows).astype(np.float32)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=None,
                    help="the reference checkout (default: $INT4GEMV_REFERENCE, else "
                         "BASELINE.json's reference_path)")
    args = ap.parse_args()
    if args.reference is None:
        sys.path.insert(0, str(REPO / "oracle"))
        import build_ref

        args.reference = build_ref.reference_dir()
    if args.reference is None or not args.reference.exists():
        raise SystemExit("no reference checkout: pass --reference or set INT4GEMV_REFERENCE")

    import torch

    sys.path.insert(0, str(args.reference))
    from int4gemv import quant as ref_quant  # the reference's own Python package
    from int4gemv import reference as ref_reference

    sys.path.insert(0, str(REPO / "oracle"))
    import build_ref

    so = build_ref.built_module() or build_ref.build(args.reference)
    spec = importlib.util.spec_from_file_location("int4gemv_ref", so)
    ref_ops = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref_ops)

    def record(name, w, m, g, keep_w, seed):
        gen = torch.Generator().manual_seed(seed)
        wt = torch.from_numpy(w)
        qw, s, z = ref_quant.quantize(wt, g)
        x = torch.randn(m, w.shape[1], generator=gen).half()
        out = {
            "group_size": np.int64(g),
            "x": x.numpy(),
            "qweight": qw.numpy(),
            "scales": s.numpy(),
            "zeros": z.numpy(),
            "y_ref": ref_reference.w4a16_reference(x, qw, s, z, g).numpy(),
            "y_seq": ref_ops.sequential(x, qw, s, z, g).numpy(),
        }
        if keep_w:
            out["w"] = w
            out["deq"] = ref_quant.dequantize(qw, s, z, g).numpy()
        np.savez_compressed(HERE / f"{name}.npz", **out)
        print(name, {k: v.shape for k, v in out.items()})

    for i, (name, m, n, k, g, keep_w) in enumerate(CASES):
        gen = torch.Generator().manual_seed(1000 + i)
        w = (torch.randn(n, k, generator=gen) * 0.02).numpy()
        record(name, w, m, g, keep_w, 2000 + i)
    record("quant_edges_g128", edge_weights(), 2, 128, True, 3000)
    record("quant_edges_g32", edge_weights(), 1, 32, True, 3001)

    # pack on values outside 0..15 (quant.py:32-37 sums q << 4j in int64, then casts to int32)
    gen = torch.Generator().manual_seed(4000)
    q = torch.randint(-40, 60, (6, 128), generator=gen, dtype=torch.int32)
    q[0, :8] = torch.tensor([2**31 - 1, -2**31, 15, 15, 15, 15, 15, 15], dtype=torch.int32)
    q[1] = torch.randint(0, 16, (128,), generator=gen, dtype=torch.int32)
    np.savez_compressed(HERE / "pack_wrap.npz", q=q.numpy(), qweight=ref_quant.pack(q).numpy())
    print("pack_wrap", tuple(q.shape))


if __name__ == "__main__":
    main()
