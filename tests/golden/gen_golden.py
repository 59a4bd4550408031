"""Generate the golden fixtures in this folder from the reference itself.

Run where a checkout of the reference source is at hand (the fixtures are
committed; the GPU tests never need the reference):

    python tests/golden/gen_golden.py --reference DIR   # or TORCH_MCPU_REFERENCE=DIR

* grouped_topk: the reference's own router function ``copied_grouped_topk``
  (tests/test_grouped_topk_compile.py:15-66 of kzwrime/torch_mcpu) is loaded
  from the reference source with ``ast`` (its module imports the compiled
  torch_mcpu extension, which is not built here) and run on CPU tensors.  On
  the reference's mcpu device every op of that function dispatches to the
  same CPU ATen kernel on a host view (csrc/aten/ops/*.cpp), except sigmoid,
  which uses the raw glibc-expf loop (unary_out.cpp:46-49); the oracle
  reproduces that loop and the tests compare the two.
* silu_and_mul / rms_norm: vLLM 0.22's native formulas
  (vllm/model_executor/layers/activation.py SiluAndMul.forward_native,
  vllm/ir/ops/layernorm.py rms_norm native impl) run on CPU.
* gated MLP: the structure of example/01_mlp_tp4/run.py:50-56,106-126
  (column-parallel gate/up, row-parallel down, SUM all-reduce) with SwiGLU,
  evaluated with torch CPU bf16 matmuls.

Rows whose reference selection is ambiguous (an exact tie in the reference's
own rounded values on a selection boundary) are recorded per fixture.
"""

from __future__ import annotations

import ast
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import configs as C  # noqa: E402

def _reference_test_file() -> str:
    """tests/test_grouped_topk_compile.py of a kzwrime/torch_mcpu checkout
    named by --reference DIR or the TORCH_MCPU_REFERENCE environment
    variable."""
    root = None
    if "--reference" in sys.argv:
        root = sys.argv[sys.argv.index("--reference") + 1]
    root = root or os.environ.get("TORCH_MCPU_REFERENCE")
    if not root:
        raise SystemExit("gen_golden.py: give the reference checkout with --reference DIR "
                         "or TORCH_MCPU_REFERENCE=DIR")
    path = os.path.join(root, "tests", "test_grouped_topk_compile.py")
    if not os.path.exists(path):
        raise SystemExit(f"gen_golden.py: {path} not found")
    return path


def load_reference_router():
    REF_TEST = _reference_test_file()
    src = open(REF_TEST).read()
    tree = ast.parse(src)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "copied_grouped_topk")
    mod = ast.Module(body=[ast.ImportFrom(module="__future__", names=[ast.alias("annotations")], level=0), fn],
                     type_ignores=[])
    ns: dict = {"torch": torch}
    exec(compile(ast.fix_missing_locations(mod), REF_TEST, "exec"), ns)
    return ns["copied_grouped_topk"]


def ambiguous_rows(gating, cfg_like, bias):
    """Rows where the reference's own values tie on a selection boundary."""
    T, E = gating.shape
    G, TG, K = cfg_like["G"], cfg_like["TG"], cfg_like["K"]
    if cfg_like["scoring"] == "sigmoid":
        scores = gating.sigmoid()
    else:
        scores = torch.softmax(gating, dim=-1)
    if bias is not None:
        keys = scores + bias.unsqueeze(0)
        gs = keys.view(T, G, -1).topk(2, dim=-1)[0].sum(-1)
    else:
        keys = scores
        gs = keys.view(T, G, -1).max(-1).values
    keys = keys.float()
    gs = gs.float()
    amb = torch.zeros(T, dtype=torch.bool)
    if TG < G:
        sg = gs.sort(-1, descending=True).values
        amb |= sg[:, TG - 1] == sg[:, TG]
    top_g = torch.topk(gs, TG, -1).indices
    mask = torch.zeros(T, G, dtype=torch.bool)
    mask.scatter_(1, top_g, True)
    # only well-defined when the group pick itself is not ambiguous
    masked = keys.masked_fill(~mask.repeat_interleave(E // G, 1), float("-inf"))
    sk = masked.sort(-1, descending=True).values
    if K < sk.shape[1]:
        amb |= sk[:, K - 1] == sk[:, K]
    return amb.numpy()


def sorted_by_id(w, ids):
    order = np.argsort(ids, axis=1, kind="stable")
    return np.take_along_axis(w, order, 1), np.take_along_axis(ids, order, 1)


def ids_digest(ids_sorted: np.ndarray, skip: np.ndarray) -> str:
    h = hashlib.sha256()
    h.update(np.ascontiguousarray(ids_sorted[~skip].astype(np.int32)).tobytes())
    return h.hexdigest()


def gen_router(fn):
    manifest = {}
    for cfg in C.ROUTER_GOLDEN + C.ROUTER_LARGE:
        gating, bias = C.router_inputs(cfg)
        hidden = torch.empty(cfg.T, 1)
        w, ids = fn(hidden, gating, topk=cfg.K, renormalize=cfg.renorm, num_expert_group=cfg.G,
                    topk_group=cfg.TG, scoring_func=cfg.scoring, routed_scaling_factor=cfg.scale,
                    e_score_correction_bias=bias)
        w = w.numpy()
        ids = ids.numpy()
        amb = ambiguous_rows(gating, dict(G=cfg.G, TG=cfg.TG, K=cfg.K, scoring=cfg.scoring), bias)
        ws, idss = sorted_by_id(w, ids)
        entry = dict(cfg=cfg.__dict__, ambiguous_rows=np.nonzero(amb)[0].tolist(),
                     ids_sorted_sha256=ids_digest(idss, amb))
        if cfg.T <= 4096:
            np.savez_compressed(os.path.join(HERE, f"router_{cfg.name}.npz"),
                                ids_sorted=idss.astype(np.int16), weights_by_id=ws,
                                ids_ref_order=ids.astype(np.int16), ambiguous=amb)
            entry["file"] = f"router_{cfg.name}.npz"
        else:
            rows = np.arange(0, cfg.T, 64)
            np.savez_compressed(os.path.join(HERE, f"router_{cfg.name}_every64.npz"),
                                rows=rows, ids_sorted=idss[rows].astype(np.int16),
                                weights_by_id=ws[rows], ambiguous=amb)
            entry["file"] = f"router_{cfg.name}_every64.npz"
        manifest[cfg.name] = entry
        print(cfg.name, "ambiguous rows:", int(amb.sum()))
    # the reference's own regression case (bf16, softmax, 8 x 16)
    hidden, gating = C.reference_test_inputs()
    w, ids = fn(hidden, gating, **C.REFERENCE_TEST_ARGS)
    a = C.REFERENCE_TEST_ARGS
    amb = ambiguous_rows(gating, dict(G=a["num_expert_group"], TG=a["topk_group"], K=a["topk"],
                                      scoring=a["scoring_func"]), None)
    ws, idss = sorted_by_id(w.numpy(), ids.numpy())
    np.savez_compressed(os.path.join(HERE, "router_reference_test_8x16_bf16.npz"),
                        ids_sorted=idss.astype(np.int16), weights_by_id=ws,
                        ids_ref_order=ids.numpy().astype(np.int16), ambiguous=amb)
    manifest["reference_test_8x16_bf16"] = dict(file="router_reference_test_8x16_bf16.npz",
                                                ambiguous_rows=np.nonzero(amb)[0].tolist())
    return manifest


def gen_bandwidth_ops():
    from vllm.ir.ops.layernorm import rms_norm
    from vllm.model_executor.layers.activation import SiluAndMul

    rms_native = rms_norm.impls["native"].impl_fn
    man = {}
    for T, d in [(64, 1024), (33, 1000), (4, 18432)]:
        x = C.silu_inputs(T, d)
        out = SiluAndMul.forward_native(x)
        name = f"silu_and_mul_T{T}_d{d}"
        np.savez_compressed(os.path.join(HERE, name + ".npz"), out_bits=out.view(torch.int16).numpy())
        man[name] = dict(T=T, d=d, file=name + ".npz")
    for T, H in [(16, 7168), (9, 4096), (8, 1000)]:
        x, w = C.rms_inputs(T, H)
        out = rms_native(x, w, C.RMS_EPS)
        name = f"rms_norm_T{T}_H{H}"
        np.savez_compressed(os.path.join(HERE, name + ".npz"), out_bits=out.view(torch.int16).numpy())
        man[name] = dict(T=T, H=H, eps=C.RMS_EPS, file=name + ".npz")
    return man


def gen_mlp():
    from vllm.ir.ops.layernorm import rms_norm
    from vllm.model_executor.layers.activation import SiluAndMul

    rms_native = rms_norm.impls["native"].impl_fn
    man = {}
    for cfg in [C.MLP_TINY, C.MLP_TINY_NORM]:
        for tp in (1, 2):
            acc = None
            for r in range(tp):
                x, rms_w, wgu, wd = C.mlp_weights(cfg, tp, r)
                h = rms_native(x, rms_w, C.RMS_EPS) if cfg.pre_norm else x
                gu = torch.mm(h, wgu.t())
                a = SiluAndMul.forward_native(gu)
                y = torch.mm(a, wd.t())
                acc = y.float() if acc is None else acc + y.float()
            out = acc.to(torch.bfloat16)
            name = f"mlp_{cfg.name}_tp{tp}"
            np.savez_compressed(os.path.join(HERE, name + ".npz"), out_bits=out.view(torch.int16).numpy())
            man[name] = dict(cfg=cfg.__dict__, tp=tp, file=name + ".npz")
    return man


def main():
    torch.set_num_threads(os.cpu_count() or 8)
    fn = load_reference_router()
    manifest = {"router": gen_router(fn)}
    manifest["bandwidth"] = gen_bandwidth_ops()
    manifest["mlp"] = gen_mlp()
    manifest["generator"] = dict(torch=torch.__version__, script="tests/golden/gen_golden.py")
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
