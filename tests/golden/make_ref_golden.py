"""Records golden vectors from GdsLLM's own CUDA kernels (needs a GPU).

The reference kernels are compiled unchanged from the reference tree into
oracle/_ref/libref_kernels.so (python oracle/build.py, in a container that
has the tree); this script runs them on seeded inputs and writes
``ref_kernels.npz`` (default: tests/golden/ref_kernels.npz, the committed
fixture).  tests/test_oracle.py checks the CPU oracle
against these outputs: dequantized values bit for bit, GEMV outputs within
the bar.

Usage: python tests/golden/make_ref_golden.py [output.npz]
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from gdsllm_b200 import synth  # noqa: E402
from oracle import reference_kernels as ref  # noqa: E402


def main(out_path: str) -> None:
    dev = torch.device("cuda", 0)
    n, k, g = 48, 1024, 128
    rec = {"affine_group": np.array(g)}

    w = synth.q4_0_weight(n, k, seed=11).to(dev)
    x = synth.activations(1, k, seed=12).to(dev)
    deq = torch.empty(n * k, dtype=torch.float16, device=dev)
    y = torch.empty(1, n, dtype=torch.float16, device=dev)
    ref.dequant_q4_0(w, deq)
    ref.gemv_q4_0(w, x, n, k, y)
    torch.cuda.synchronize()
    rec.update(q4_0_w=w.cpu().numpy(), q4_0_x=x.cpu().numpy(), q4_0_dequant=deq.cpu().numpy(),
               q4_0_gemv=y.cpu().numpy(), q4_0_shape=np.array([n, k]))

    w = synth.q8_0_weight(n, k, seed=13).to(dev)
    x = synth.activations(1, k, seed=14).to(dev)
    ref.dequant_q8_0(w, deq)
    ref.gemv_q8_0(w, x, n, k, y)
    torch.cuda.synchronize()
    rec.update(q8_0_w=w.cpu().numpy(), q8_0_x=x.cpu().numpy(), q8_0_dequant=deq.cpu().numpy(),
               q8_0_gemv=y.cpu().numpy(), q8_0_shape=np.array([n, k]))

    words, s, b = (t.to(dev) for t in synth.affine_q4_weight(n, k, group=g, seed=15))
    x = synth.activations(1, k, seed=16).to(dev)
    ref.dequant_affine_q4(words, s, b, k, g, deq)
    ref.gemv_affine_q4(words, s, b, x, n, k, g, y)
    torch.cuda.synchronize()
    rec.update(affine_words=words.cpu().numpy().view(np.uint32), affine_scales=s.cpu().numpy(),
               affine_biases=b.cpu().numpy(), affine_x=x.cpu().numpy(),
               affine_dequant=deq.cpu().numpy(), affine_gemv=y.cpu().numpy(),
               affine_shape=np.array([n, k]))

    Path(out_path).parent.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out_path, **rec)
    print("wrote", out_path)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(ROOT / "tests" / "golden" / "ref_kernels.npz"))
