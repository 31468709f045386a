"""Generate the golden fixtures in this folder from the reference itself.

Runs ZHANGWENTAI/PASA's ``pisa_pg_attention``
(``svg/kernels/triton/group_pisa_attention.py:307-398``) on CPU through the
Triton interpreter and stores its intermediate and final outputs.  Only the
fp32 path is meaningful under the interpreter (it keeps bf16 tensors as raw
uint16 and would add bit patterns), so every case here is fp32.

Inputs are not stored: they are regenerated from the seed with torch's CPU
generator (:func:`case_inputs`), and a SHA-256 of their bytes is stored so
that a changed random stream is detected instead of silently compared.

Usage (in a container that has the reference checkout):

    python tests/golden/make_golden.py /path/to/reference

The reference module is loaded by file path, so ``svg/__init__.py`` (which
patches FlashInfer) and the model modules are never imported.  Two in-process
shims make it run on CPU: ``supports_host_descriptor`` returns True, and the
autotuner around ``fused_chunk_reduce_kernel`` is unwrapped (autotuning needs
a GPU timer).
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent

# name, B, H, T, D, density, seed, kind, extra
CASES = [
    # 1 batch, 4 heads, D 64, 1024 tokens, top-25% blocks
    dict(name="tiny", B=1, H=4, T=1024, D=64, density=0.25, seed=0, kind="normal"),
    # ragged last block (1000 = 15*64 + 40)
    dict(name="ragged", B=1, H=1, T=1000, D=64, density=0.3, seed=1, kind="normal"),
    # partial last group (NT=40 -> 2 groups) and a 4-token last block
    dict(name="partial_group", B=1, H=1, T=2500, D=64, density=0.15, seed=2, kind="normal"),
    # head_dim 128, batch 2
    dict(name="d128", B=2, H=1, T=640, D=128, density=0.2, seed=3, kind="normal"),
    # keys built so that zero-order logits exceed the exact-phase maximum:
    # exercises the running-max update inside the correction phase
    dict(name="max_shift", B=1, H=1, T=2200, D=64, density=0.25, seed=4, kind="max_shift"),
    # selection noise (use_random=True); the drawn noise is stored
    dict(name="random_bias", B=1, H=1, T=1024, D=64, density=0.2, seed=5, kind="normal",
         use_random=True),
    # plain dot-product selection (use_cov_bias=False)
    dict(name="no_cov_bias", B=1, H=1, T=960, D=64, density=0.25, seed=6, kind="normal",
         use_cov_bias=False),
    # a single selected block per query block (NS = 1)
    dict(name="ns_one", B=1, H=1, T=640, D=64, density=0.01, seed=7, kind="normal"),
    # every block selected (NS = NT): the correction phase sees only masks
    dict(name="ns_all", B=1, H=1, T=700, D=64, density=1.0, seed=8, kind="normal"),
]


def case_inputs(case):
    """Seeded fp32 q, k, v of shape [B, H, T, D] (torch CPU generator)."""
    import torch

    g = torch.Generator().manual_seed(int(case["seed"]))
    shape = (case["B"], case["H"], case["T"], case["D"])
    q = torch.randn(shape, generator=g, dtype=torch.float32)
    k = torch.randn(shape, generator=g, dtype=torch.float32)
    v = torch.randn(shape, generator=g, dtype=torch.float32)
    if case["kind"] == "max_shift":
        # odd blocks of the second 32-block group: nearly constant keys c * e
        # (small covariance norm, so the top-k skips them, and large mean
        # logits, so the running max grows in the correction phase after the
        # first group has already added to g_l); all other keys N(0,1)
        D, T = case["D"], case["T"]
        e = torch.randn(D, generator=g, dtype=torch.float32)
        e = e / e.norm() * (D ** 0.5)
        nt = -(-T // 64)
        for j in range(33, nt, 2):
            c = 2.0 + 3.0 * torch.rand(1, generator=g).item()
            rows = slice(j * 64, min(T, (j + 1) * 64))
            k[:, :, rows, :] = c * e + 0.01 * k[:, :, rows, :]
    return q, k, v


def input_digest(q, k, v) -> str:
    h = hashlib.sha256()
    for t in (q, k, v):
        h.update(t.contiguous().numpy().tobytes())
    return h.hexdigest()


def load_reference(ref_root: Path):
    os.environ["TRITON_INTERPRET"] = "1"
    path = ref_root / "svg" / "kernels" / "triton" / "group_pisa_attention.py"
    spec = importlib.util.spec_from_file_location("pasa_reference_group_pisa", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.supports_host_descriptor = lambda: True
    mod.fused_chunk_reduce_kernel = mod.fused_chunk_reduce_kernel.fn
    return mod


def run_case(mod, case):
    import numpy as np
    import torch

    q, k, v = case_inputs(case)
    B, H, T, D = q.shape
    block, group = 64, 32
    scale = D ** -0.5
    use_cov_bias = case.get("use_cov_bias", True)
    use_random = case.get("use_random", False)

    # intermediates, through the reference's own helpers
    qc, kc, vc, hc, h_norm = mod.fused_chunk_reduce(q, k, v, block)
    h_group, n_groups = mod.compute_h_group(hc, group)

    # the op; for use_random the global CPU generator is seeded so the noise
    # draw inside the reference is reproducible, and the same draw is
    # repeated here to store it
    noise = None
    if use_random:
        torch.manual_seed(1000 + int(case["seed"]))
        noise = torch.randn_like(torch.log(h_norm + 1e-6))
        torch.manual_seed(1000 + int(case["seed"]))
    o = mod.pisa_pg_attention(q, k, v, density=case["density"], block_size=block,
                              group_size=group, use_cov_bias=use_cov_bias,
                              use_random=use_random)

    # the selection, restated from :365-375 with the same torch calls, to
    # store the indices the op used
    score = torch.einsum("bhid, bhjd -> bhij", qc, kc * scale)
    if use_cov_bias:
        log_bias = torch.log(h_norm + 1e-6)
        if use_random:
            log_bias = log_bias + noise
        score = score + log_bias.unsqueeze(2)
    NT = -(-T // block)
    top_k = min(max(1, int(case["density"] * NT)), NT)
    indices = torch.topk(score, k=top_k, dim=-1).indices.reshape(B * H, NT, top_k).to(torch.int32)

    out = dict(
        o=o.numpy(), qc=qc.reshape(B * H, NT, D).numpy(), kc=kc.reshape(B * H, NT, D).numpy(),
        vc=vc.reshape(B * H, NT, D).numpy(), h_norm=h_norm.reshape(B * H, NT).numpy(),
        h_group=h_group.numpy(), indices=indices.numpy(),
        score=score.reshape(B * H, NT, NT).numpy(),
    )
    if noise is not None:
        out["noise"] = noise.reshape(B * H, NT).numpy()
    meta = dict(case, digest=input_digest(q, k, v), top_k=top_k, n_groups=int(n_groups))
    return out, meta


def main(argv):
    import numpy as np

    ref_root = Path(argv[1] if len(argv) > 1 else "/root/reference")
    mod = load_reference(ref_root)
    manifest = {}
    for case in CASES:
        out, meta = run_case(mod, case)
        np.savez_compressed(HERE / f"{case['name']}.npz", **out)
        manifest[case["name"]] = meta
        print(case["name"], {k: v.shape for k, v in out.items()})
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main(sys.argv)
