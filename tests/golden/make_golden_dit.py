"""Generate ``dit_rows.npz`` in this folder from the reference itself.

Runs ZHANGWENTAI/PASA's row kernels of the DiT block on CPU through the
Triton interpreter (fp32, the only dtype the interpreter handles correctly):

* ``triton_layernorm_forward`` without / with affine
  (svg/kernels/triton/layernorm.py:13-218),
* ``triton_rmsnorm_forward`` (rmsnorm.py:8-100),
* ``triton_modulate_shift_forward`` and
  ``triton_modulate_gate_residual_forward`` (modulate.py:12-164),

and the rotary embedding's torch path (svg/models/wan/attention.py:49-57,
the nested ``_apply_rotary_emb``), taken from the source file with ``ast``
and executed as written, on bf16 input (pure torch, so bf16 is exact on CPU).

Inputs are regenerated from seeds with torch's CPU generator; their SHA-256
is stored to detect a changed random stream.

Usage (in a container that has the reference checkout):

    python tests/golden/make_golden_dit.py /path/to/reference
"""
from __future__ import annotations

import ast
import hashlib
import importlib.util
import json
import os
import sys
import types
from pathlib import Path

HERE = Path(__file__).resolve().parent

# (name, rows, cols): cols <= 512 runs the reference's 32-row programs (rows
# must be a multiple of 32, the kernels do not mask rows); larger cols one
# row per program with the columns padded to a power of two
ROW_CASES = [("n320", 32, 320), ("n640", 9, 640)]
ROPE_CASE = dict(heads=3, frames=2, height=3, width=4, head_dim=32, seed=11)
EPS = 1e-6


def row_inputs(rows, cols, seed):
    import torch

    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(s, generator=g, dtype=torch.float32)
    return dict(x=r(1, rows, cols) * 3 + 0.5, add=r(1, rows, cols), w=1 + 0.1 * r(cols), b=0.1 * r(cols),
                scale=0.2 * r(cols), shift=0.2 * r(cols), gate=r(cols))


def rope_inputs(c):
    import torch

    g = torch.Generator().manual_seed(c["seed"])
    L = c["frames"] * c["height"] * c["width"]
    return torch.randn((1, c["heads"], L, c["head_dim"]), generator=g).to(torch.bfloat16)


def digest(*ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(t.contiguous().view(-1).view(__import__("torch").uint8).numpy().tobytes())
    return h.hexdigest()


def load_triton_package(ref_root: Path):
    os.environ["TRITON_INTERPRET"] = "1"
    tdir = ref_root / "svg" / "kernels" / "triton"
    pkg = types.ModuleType("pasa_ref_triton")
    pkg.__path__ = [str(tdir)]
    sys.modules["pasa_ref_triton"] = pkg
    mods = {}
    for name in ("utils", "layernorm", "rmsnorm", "modulate"):
        spec = importlib.util.spec_from_file_location(f"pasa_ref_triton.{name}", tdir / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = mod
        spec.loader.exec_module(mod)
        mods[name] = mod
    return mods


def load_rope_fallback(ref_root: Path):
    """The nested ``_apply_rotary_emb`` of attention.py's torch fallback."""
    import torch

    src = (ref_root / "svg" / "models" / "wan" / "attention.py").read_text()
    for node in ast.walk(ast.parse(src)):
        if isinstance(node, ast.FunctionDef) and node.name == "_apply_rotary_emb":
            ns = {"torch": torch}
            exec(compile(ast.Module(body=[node], type_ignores=[]), "attention.py", "exec"), ns)
            return ns["_apply_rotary_emb"], node.lineno
    raise RuntimeError("_apply_rotary_emb not found")


def main(argv):
    import numpy as np
    import torch

    sys.path.insert(0, str(HERE.parents[1]))
    from oracle.dit_oracle import rope_table

    ref_root = Path(argv[1] if len(argv) > 1 else "/root/reference")
    m = load_triton_package(ref_root)
    out, meta = {}, {}
    for i, (name, rows, cols) in enumerate(ROW_CASES):
        t = row_inputs(rows, cols, 100 + i)
        ln = m["layernorm"].triton_layernorm_forward(t["x"], None, None, EPS, elementwise_affine=False)
        lnp = m["layernorm"].triton_layernorm_forward(t["x"], t["w"], t["b"], EPS, elementwise_affine=True)
        rms = m["rmsnorm"].triton_rmsnorm_forward(t["x"], t["w"], EPS)
        mod = m["modulate"].triton_modulate_shift_forward(ln, t["scale"], t["shift"], output_dtype=torch.float32)
        res = m["modulate"].triton_modulate_gate_residual_forward(t["x"], t["add"], t["gate"],
                                                                  output_dtype=torch.float32)
        for k, v in dict(ln=ln, ln_affine=lnp, rms=rms, modulate=mod, gate_residual=res).items():
            out[f"{name}_{k}"] = v.reshape(rows, cols).numpy()
        meta[name] = dict(rows=rows, cols=cols, seed=100 + i, digest=digest(*t.values()))

    fn, line = load_rope_fallback(ref_root)
    c = ROPE_CASE
    x = rope_inputs(c)
    cos, sin = rope_table(c["frames"], c["height"], c["width"], c["head_dim"])
    # the complex table the model passes: cos + i sin, float64
    freqs = torch.complex(torch.from_numpy(cos), torch.from_numpy(sin))
    y = fn(x, freqs[None, None])
    out["rope_out_bits"] = y.view(torch.int16).numpy()
    meta["rope"] = dict(c, digest=digest(x), source_line=line)
    np.savez_compressed(HERE / "dit_rows.npz", **out)
    (HERE / "dit_rows.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main(sys.argv)
