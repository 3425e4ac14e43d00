"""Generate tests/golden/checkpoint_*.npz: AWQ and GPTQ checkpoint tensors made by a third-party
packer (vLLM 0.22, vllm/model_executor/layers/quantization/utils/quant_utils.py: awq_pack,
gptq_pack, pack_cols) from weights quantised by the REFERENCE (int4gemv/quant.py:14-29).

Run in the build container, where the reference checkout and vLLM exist:

    python tests/golden/make_checkpoint_golden.py [--reference PATH]

Each file holds the reference's (qweight, scales, zeros) and the same weights as
  awq_qweight [K, N/8], awq_qzeros [K/g, N/8], awq_scales [K/g, N]
  gptq_qweight [K/8, N], gptq_qzeros ("gptq": zeros minus one), gptq_v2_qzeros (zeros as they are),
  gptq_scales [K/g, N]
so that the oracle's format restatement and the repack kernels are pinned to an independent packer.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]

CASES = [("checkpoint_n64_k512_g128", 64, 512, 128, 5000),
         ("checkpoint_n48_k256_g32", 48, 256, 32, 5001)]


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
    from vllm.model_executor.layers.quantization.utils.quant_utils import (awq_pack, gptq_pack,
                                                                           pack_cols)

    sys.path.insert(0, str(args.reference))
    from int4gemv import quant as ref_quant  # the reference's own Python package

    for name, n, k, g, seed in CASES:
        gen = torch.Generator().manual_seed(seed)
        w = torch.randn(n, k, generator=gen) * 0.02
        w[0] = w[0].abs() + 0.01   # all-positive groups: zero point 0 (stored as 15 by "gptq")
        w[1] = -w[1].abs() - 0.01  # all-negative groups: zero point 15
        qw, s, z = ref_quant.quantize(w, g)
        q = ref_quant.unpack(qw)                       # [N, K] int32
        zi = z.float().round().to(torch.int32)         # [N, K/g]
        qt, zt = q.t().contiguous(), zi.t().contiguous()  # [K, N], [K/g, N]
        out = {
            "group_size": np.int64(g),
            "qweight": qw.numpy(), "scales": s.numpy(), "zeros": z.numpy(),
            "awq_qweight": awq_pack(qt, 4, k, n).numpy(),
            "awq_qzeros": awq_pack(zt, 4, k // g, n).numpy(),
            "awq_scales": s.t().contiguous().numpy(),
            "gptq_qweight": gptq_pack(qt, 4, k, n).numpy(),
            "gptq_qzeros": pack_cols((zt - 1) & 0xF, 4, k // g, n).numpy(),
            "gptq_v2_qzeros": pack_cols(zt, 4, k // g, n).numpy(),
            "gptq_scales": s.t().contiguous().numpy(),
        }
        np.savez_compressed(HERE / f"{name}.npz", **out)
        print(name, {key: v.shape for key, v in out.items()})


if __name__ == "__main__":
    main()
