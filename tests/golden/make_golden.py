"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a container where the reference checkout is present (it is not on the
GPU box; the committed .npz files travel instead):

    TRITON_INTERPRET=1 python tests/golden/make_golden.py REFERENCE_ROOT

* ``dsv4_a100_patch/triton_kernels/mxfp4_int8_moe.py`` is loaded standalone
  with importlib (its package __init__ needs SGLang).  Its CPU torch quantiser,
  its torch repack and its remap statistics run on CPU directly; its Triton
  repack kernels run under Triton's CPU interpreter (``TRITON_INTERPRET=1``).
* ``_dequant_mxfp4`` / ``_mxfp4_moe_reference`` / ``_relative_l2`` are pulled
  out of ``tests/test_mxfp4_int8_moe.py`` with ``ast`` (that module imports the
  SGLang-dependent package at top level).

Inputs come from ``tests/gen_inputs.py`` (CPU generators); each fixture also
stores its inputs or, for the larger config-1 case, a checksum of them.
"""

from __future__ import annotations

import ast
import hashlib
import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
import gen_inputs as G  # noqa: E402


def load_reference(root: Path):
    if os.environ.get("TRITON_INTERPRET") != "1":
        raise SystemExit("set TRITON_INTERPRET=1 so the Triton repack runs on CPU")
    path = root / "dsv4_a100_patch/triton_kernels/mxfp4_int8_moe.py"
    spec = importlib.util.spec_from_file_location("ref_pymoe", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_pymoe"] = mod
    spec.loader.exec_module(mod)
    test_src = (root / "tests/test_mxfp4_int8_moe.py").read_text()
    tree = ast.parse(test_src)
    keep = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in (
            "_dequant_mxfp4", "_mxfp4_moe_reference", "_relative_l2"):
            keep.append(node)
        if isinstance(node, ast.Assign) and any(
                isinstance(t, ast.Name) and t.id == "_LUT_X2" for t in node.targets):
            keep.append(node)
    ns = {"torch": torch}
    exec(compile(ast.Module(body=keep, type_ignores=[]), "ref_test_helpers", "exec"), ns)
    return mod, ns


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main():
    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DSV4_REFERENCE_ROOT")
    if not arg:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (or set DSV4_REFERENCE_ROOT)")
    root = Path(arg)
    ref, helpers = load_reference(root)
    out = {}

    # quantiser: reference test shape 17x129, row 0 zero (TEST_MOE:137-150)
    for name, dt in (("f32", torch.float32), ("f16", torch.float16), ("bf16", torch.bfloat16)):
        gen = torch.Generator()
        gen.manual_seed(20260622)
        a = (torch.randn((17, 129), generator=gen) * 0.5).to(dt)
        a[0].zero_()
        q, s = ref.quantize_per_token_int8(a, 0.0)
        np.savez(HERE / f"quant_{name}.npz", a=a.float().numpy(), q=q.numpy(), scale=s.numpy(),
                 clamp=np.float32(0.0))
    gen = torch.Generator()
    gen.manual_seed(7)
    a = (torch.randn((9, 300), generator=gen) * 2.0).to(torch.bfloat16)
    q, s = ref.quantize_per_token_int8(a, 1.5)
    np.savez(HERE / "quant_clamp.npz", a=a.float().numpy(), q=q.numpy(), scale=s.numpy(),
             clamp=np.float32(1.5))

    # repack, both backends (TEST_MOE:123-134 inputs, plus a BASELINE-range case)
    cases = {
        "repack_span3": dict(e=3, n=19, k=128, seed=20260620, exp_range=None),
        "repack_baseline": dict(e=2, n=40, k=256, seed=99, exp_range=(-8, -4)),
        "repack_wide": dict(e=2, n=16, k=128, seed=5, exp_range=(-20, 0)),
    }
    for name, c in cases.items():
        w, s = G.make_random_packed_mxfp4(c["e"], c["n"], c["k"], c["seed"], exp_range=c["exp_range"])
        tri = ref._remap_mxfp4_weight_for_int8_triton(w, s, headroom_bits=3)
        tor = ref.remap_mxfp4_weight_for_int8(w, s, headroom_bits=3, use_triton=False)
        np.savez(HERE / f"{name}.npz", weight=w.numpy(), scale=s.numpy(),
                 tri_b=tri[0].numpy(), tri_shift=tri[1].numpy(), tri_cs=tri[2].numpy(),
                 torch_b=tor[0].numpy(), torch_shift=tor[1].numpy(), torch_cs=tor[2].numpy())

    # remap statistics (TEST_MOE:111-120)
    w, s = G.make_random_packed_mxfp4(3, 96, 128, 20260618)
    st = ref._compute_remap_stats(w, s, headroom_bits=3)
    np.savez(HERE / "remap_stats.npz", weight=w.numpy(), scale=s.numpy(),
             overflow_count=st["overflow_count"], exact_rate_nonzero=st["exact_rate_nonzero"],
             mean_rel_err_nonzero=st["mean_rel_err_nonzero"], row_span_max=st["row_span_max"])

    # float reference MoE, reference test shape (TEST_MOE:165-258)
    e, t, h, i, topk = 4, 13, 128, 128, 2
    w13, s13 = G.make_random_packed_mxfp4(e, 2 * i, h, 21)
    w2, s2 = G.make_random_packed_mxfp4(e, h, i, 22)
    ids = G.round_robin_routing(t, e, topk)
    gen = torch.Generator()
    gen.manual_seed(20260621)
    tw = torch.softmax(torch.randn(t, topk, generator=gen), dim=-1)
    x = G.randn_bf16((t, h), 23, 0.2)
    ref_out = helpers["_mxfp4_moe_reference"](x, w13, s13, w2, s2, ids, tw)
    np.savez(HERE / "moe_ref_small.npz", w13=w13.numpy(), s13=s13.numpy(), w2=w2.numpy(),
             s2=s2.numpy(), topk_ids=ids.numpy(), topk_weights=tw.numpy(),
             hidden_bits=x.view(torch.int16).numpy(), out_bits=ref_out.view(torch.int16).numpy())

    # BASELINE config 1 (CPU reference MoE): H=1024, I=512, E=8, top-2 softmax, T=16
    e, t, h, i, topk = 8, 16, 1024, 512, 2
    w13, s13 = G.make_random_packed_mxfp4(e, 2 * i, h, 101, exp_range=(-8, -4))
    w2, s2 = G.make_random_packed_mxfp4(e, h, i, 102, exp_range=(-8, -4))
    ids, tw = G.routing_softmax_topk(t, e, topk, 103)
    x = G.randn_bf16((t, h), 104, 1.0)
    ref_out = helpers["_mxfp4_moe_reference"](x, w13, s13, w2, s2, ids, tw)
    np.savez(HERE / "moe_ref_config1.npz",
             input_sha=sha(w13.numpy(), s13.numpy(), w2.numpy(), s2.numpy(), ids.numpy(),
                           tw.numpy(), x.view(torch.int16).numpy()),
             out_bits=ref_out.view(torch.int16).numpy())

    # dense reference (TEST_MOE:153-162)
    n, k, m = 128, 128, 11
    w, s = G.make_random_packed_mxfp4(1, n, k, 20260619)
    x = G.randn_bf16((m, k), 31, 0.2)
    ref_w = helpers["_dequant_mxfp4"](w, s).reshape(1, n, k)[0]
    ref_d = torch.matmul(x.float(), ref_w.float().t()).to(torch.bfloat16)
    np.savez(HERE / "dense_ref.npz", weight=w[0].numpy(), scale=s[0].numpy(),
             x_bits=x.view(torch.int16).numpy(), out_bits=ref_d.view(torch.int16).numpy())
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
