"""Records golden outputs of GdsLLM's own MoE decode code (moe_mlp_selective,
gdsllm/runtime/qwen_moe.py:419-516) on seeded inputs.

The reference module is imported from the reference tree given on the
command line and run on CPU tensors.  Its fused affine-Q4 GEMV
(_fused_affine_q4_gemv, a CUDA op) is replaced by the oracle's CPU GEMV
(dequantize, fp32 matmul, fp16), so the fixture pins everything around the
GEMVs: SiLU and product rounding, the per-slot fp16 routing-weighted sum,
the shared expert and its sigmoid gate, and the final clamp.
tests/test_oracle.py checks oracle.moe_mlp_reference against it bit for bit.

Usage: python tests/golden/make_moe_golden.py <reference-tree> [out.npz]
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from gdsllm_b200 import synth  # noqa: E402

EXPERTS, HIDDEN, INTER, GROUP, TOP_K, NTOK = 6, 256, 128, 32, 3, 3


def main(ref_tree: str, out_path: str) -> None:
    sys.path.insert(0, ref_tree)
    from gdsllm.runtime import qwen_moe as qm

    def stack(rows, cols, seed, experts=EXPERTS):
        return tuple(t.numpy() for t in synth.affine_q4_weight(rows, cols, group=GROUP, seed=seed,
                                                               lead=(experts,)))

    gate, up, down = stack(INTER, HIDDEN, 1), stack(INTER, HIDDEN, 2), stack(HIDDEN, INTER, 3)
    sgate, sup, sdown = stack(INTER, HIDDEN, 4, 1), stack(INTER, HIDDEN, 5, 1), stack(HIDDEN, INTER, 6, 1)
    x = synth.activations(NTOK, HIDDEN, seed=7).numpy()
    g = torch.Generator().manual_seed(8)
    ids = np.stack([torch.randperm(EXPERTS, generator=g)[:TOP_K].numpy() for _ in range(NTOK)])
    route_w = torch.softmax(torch.randn(NTOK, TOP_K, generator=g), -1).half().numpy()
    sg_w = (torch.randn(1, HIDDEN, generator=g) / HIDDEN ** 0.5).half().numpy()

    def meta(st, e):
        return {"quant_type": "affine_q4", "w16": oracle.expert_f16(st, e, GROUP)}

    def cpu_gemv(xv, m):  # stands in for the CUDA op, same shapes as qwen_moe.py:38-55
        y = oracle.gemv_cpu(m["w16"], xv.reshape(-1).numpy())
        return torch.from_numpy(y).unsqueeze(0)

    qm._fused_affine_q4_gemv = cpu_gemv
    experts = {}
    for e in range(EXPERTS):
        experts[f"gate_proj.{e}"] = meta(gate, e)
        experts[f"up_proj.{e}"] = meta(up, e)
        experts[f"down_proj.{e}"] = meta(down, e)
    weights = {
        "mlp.shared_expert.gate_proj.weight": meta(sgate, 0),
        "mlp.shared_expert.up_proj.weight": meta(sup, 0),
        "mlp.shared_expert.down_proj.weight": meta(sdown, 0),
        "mlp.shared_expert_gate.weight": torch.from_numpy(sg_w),
    }
    outs = []
    for t in range(NTOK):  # the decode branch handles one token per call
        xt = torch.from_numpy(x[t]).view(1, 1, HIDDEN)
        y = qm.moe_mlp_selective(xt, weights, experts, torch.from_numpy(ids[t]).long().view(1, 1, TOP_K),
                                 torch.from_numpy(route_w[t]).view(1, 1, TOP_K), TOP_K)
        outs.append(y.reshape(-1).numpy())
    rec = {"group": np.array(GROUP), "x": x, "ids": ids.astype(np.int32), "route_w": route_w,
           "shared_gate_w": sg_w, "y": np.stack(outs)}
    for name, st in (("gate", gate), ("up", up), ("down", down), ("sgate", sgate), ("sup", sup),
                     ("sdown", sdown)):
        rec[f"{name}_w"], rec[f"{name}_s"], rec[f"{name}_b"] = st
    np.savez_compressed(out_path, **rec)
    print("wrote", out_path, {k: v.shape for k, v in rec.items()})


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else str(ROOT / "tests/golden/moe_decode.npz"))
