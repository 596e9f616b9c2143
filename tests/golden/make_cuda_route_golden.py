"""Record the reference router's results as torch computes them on a CUDA GPU.

The reference routes with three torch calls (nanovllm/layers/moe.py:872-878):
    probs = F.softmax(logits, dim=-1, dtype=torch.float32)
    w, ids = torch.topk(probs, k, dim=-1)
    w /= w.sum(dim=-1, keepdim=True)          # norm_topk_prob
    w = w.to(torch.bfloat16)
On a GPU these are torch's CUDA kernels, whose order for equal probabilities
(frequent with bf16 logits) differs from the CPU kernels that
make_golden.py records.  This script runs exactly those calls on cuda:0 over
seeded logit sets with many ties and writes, per set, the inputs, the fp32
probabilities (for rows with a tie in their top k + 1, capped), the ids and
the bf16 weight bits to route_cuda_golden.npz.  tests/test_oracle_golden.py
pins the oracle's selection and renormalisation to it on the CPU.

Usage (on a machine with a CUDA GPU):
    python tests/golden/make_cuda_route_golden.py [--out PATH]
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import extend_nano_vllm_b200.workloads as wl  # noqa: E402

MAX_PROB_ROWS = 384


def logit_sets() -> dict[str, tuple[torch.Tensor, int]]:
    """name -> (logits on the CPU, top_k).  Every set is seeded."""
    golden = np.load(os.path.join(HERE, "moe_golden.npz"))
    sets = {}
    sets["bf16_gold256"] = (torch.from_numpy(golden["route_bf16_logits"].astype(np.int16))
                            .view(torch.bfloat16).reshape(256, 128), 8)
    sets["bf16_zipf8192"] = (wl.zipf_logits(8192, 128, seed=41).to(torch.bfloat16), 8)
    g = torch.Generator().manual_seed(43)
    # Coarsely quantised fp32 logits: ties among distinct experts at any k.
    sets["f32_q_e40_k6"] = ((torch.randn((256, 40), generator=g) * 4).round() / 4, 6)
    sets["f32_q_e8_k2"] = ((torch.randn((256, 8), generator=g) * 2).round() / 2, 2)
    sets["f32_q_e64_k32"] = ((torch.randn((128, 64), generator=g) * 2).round() / 2, 32)
    sets["f32_q_e1024_k8"] = ((torch.randn((32, 1024), generator=g) * 8).round() / 8, 8)
    sets["bf16_q_e128_k5"] = (((torch.randn((256, 128), generator=g) * 4).round() / 4)
                              .to(torch.bfloat16), 5)
    return {k: (v[0].contiguous(), v[1]) for k, v in sets.items()}


def cuda_route(logits: torch.Tensor, top_k: int, renormalize: bool = True):
    """The reference's _route arithmetic (moe.py:872-878) on the logits' device."""
    probs = F.softmax(logits, dim=-1, dtype=torch.float32)
    w, ids = torch.topk(probs, top_k, dim=-1)
    if renormalize:
        w /= w.sum(dim=-1, keepdim=True)
    return probs, w.to(torch.bfloat16), ids


def tie_rows(probs: np.ndarray, top_k: int) -> np.ndarray:
    top = -np.sort(-probs, axis=-1)[:, : top_k + 1]
    return np.nonzero(np.any(top[:, 1:] == top[:, :-1], axis=-1))[0]


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--out", default=os.path.join(HERE, "route_cuda_golden.npz"))
    args = parser.parse_args()
    if not torch.cuda.is_available():
        raise SystemExit("a CUDA GPU is required")
    out = {"torch_version": np.array(torch.__version__),
           "device": np.array(torch.cuda.get_device_name(0))}
    for name, (logits, k) in logit_sets().items():
        probs, w, ids = cuda_route(logits.cuda(), k)
        probs = probs.cpu().numpy()
        rows = tie_rows(probs, k)[:MAX_PROB_ROWS]
        out[f"{name}_k"] = np.array(k)
        if logits.dtype == torch.bfloat16:
            out[f"{name}_logits_bf16"] = logits.view(torch.int16).numpy().view(np.uint16)
        else:
            out[f"{name}_logits_f32"] = logits.numpy()
        out[f"{name}_tie_rows"] = rows.astype(np.int32)
        out[f"{name}_tie_probs"] = probs[rows]
        out[f"{name}_ids"] = ids.cpu().numpy().astype(np.int16)
        out[f"{name}_w"] = w.cpu().view(torch.int16).numpy().view(np.uint16)
        print(f"{name}: {logits.shape[0]} rows, k={k}, {len(tie_rows(probs, k))} tie rows")
    if "bf16_zipf8192_logits_bf16" in out:
        # Regenerated from its seed by the tests; not stored.
        del out["bf16_zipf8192_logits_bf16"]
    np.savez_compressed(args.out, **out)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
