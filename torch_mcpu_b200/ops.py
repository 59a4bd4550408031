"""Python surface of the hot-path ops, mirroring the reference's interface.

Tensors are torch tensors resident on the B200 (device "cuda"); every op is
enqueued on torch's current CUDA stream and returns without synchronising,
like the reference's mcpu ops, which return after enqueueing on the current
mcpu stream.  Each call goes straight to the C-ABI of include/mcpu_ops.h.
"""

from __future__ import annotations

import torch

from . import _lib

_DTYPES = {torch.float32: 0, torch.bfloat16: 1}
_SCORING = {"softmax": 0, "sigmoid": 1}


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_device(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a device tensor (got device {t.device}); "
                           "the mcpu B200 ops have no CPU fallback")


def grouped_topk(
    hidden_states: torch.Tensor,
    gating_output: torch.Tensor,
    topk: int,
    renormalize: bool,
    num_expert_group: int,
    topk_group: int,
    scoring_func: str = "softmax",
    routed_scaling_factor: float = 1.0,
    e_score_correction_bias: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused grouped top-k router; same arguments and outputs as the
    reference's copied_grouped_topk (tests/test_grouped_topk_compile.py:15-26):
    returns (topk_weights float32 [T, topk], topk_ids int32 [T, topk])."""
    if hidden_states.size(0) != gating_output.size(0):
        raise AssertionError("Number of tokens mismatch")
    if scoring_func not in _SCORING:
        raise ValueError(f"Unsupported scoring function: {scoring_func}")
    _require_device(gating_output, "gating_output")
    if gating_output.dim() != 2:
        raise RuntimeError("grouped_topk: gating_output must be [num_tokens, num_experts]")
    if gating_output.dtype not in _DTYPES:
        raise RuntimeError(f"grouped_topk: unsupported gating dtype {gating_output.dtype}")
    g = gating_output.contiguous()
    T, E = g.shape
    bias = None
    if e_score_correction_bias is not None:
        _require_device(e_score_correction_bias, "e_score_correction_bias")
        if e_score_correction_bias.numel() != E:
            raise RuntimeError("grouped_topk: e_score_correction_bias must have num_experts elements")
        bias = e_score_correction_bias.to(torch.float32).contiguous()
    w = torch.empty(T, topk, dtype=torch.float32, device=g.device)
    ids = torch.empty(T, topk, dtype=torch.int32, device=g.device)
    lib = _lib.load()
    rc = lib.mcpu_grouped_topk(
        g.data_ptr(), _DTYPES[g.dtype], T, E, num_expert_group, topk_group, topk,
        int(bool(renormalize)), float(routed_scaling_factor),
        None if bias is None else bias.data_ptr(), _SCORING[scoring_func],
        w.data_ptr(), ids.data_ptr(), _stream_handle(g.device),
    )
    _lib.check(rc, "grouped_topk")
    return w, ids


def grouped_topk_exact_rows(reset: bool = False) -> int:
    """Rows resolved on the router's exact near-tie path (diagnostics)."""
    import ctypes

    n = ctypes.c_ulonglong(0)
    _lib.check(_lib.load().mcpu_grouped_topk_exact_rows(ctypes.byref(n), int(reset)),
               "grouped_topk_exact_rows")
    return int(n.value)


def silu_and_mul(out: torch.Tensor, x: torch.Tensor) -> None:
    """mcpu::silu_and_mul(Tensor(a!) out, Tensor x) -> (): out = silu(x[..., :d]) * x[..., d:]
    (vLLM SiluAndMul, activation.py:118-140), bf16."""
    _require_device(x, "x")
    _require_device(out, "out")
    d = x.shape[-1] // 2
    if x.shape[-1] != 2 * d or tuple(out.shape) != tuple(x.shape[:-1]) + (d,):
        raise RuntimeError(f"silu_and_mul: out must be {tuple(x.shape[:-1]) + (d,)}, got {tuple(out.shape)}")
    if x.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise RuntimeError("silu_and_mul: bfloat16 tensors expected")
    if not (x.is_contiguous() and out.is_contiguous()):
        raise RuntimeError("silu_and_mul: contiguous tensors expected")
    T = x.numel() // max(1, x.shape[-1])
    _lib.check(_lib.load().mcpu_silu_and_mul(out.data_ptr(), x.data_ptr(), T, d, 1,
                                             _stream_handle(x.device)), "silu_and_mul")


def rms_norm(out: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, eps: float) -> None:
    """mcpu::rms_norm(Tensor(a!) out, Tensor x, Tensor weight, float eps) -> ()
    (vLLM rms_norm native, vllm/ir/ops/layernorm.py:10-21), bf16."""
    for t, n in ((x, "x"), (out, "out"), (weight, "weight")):
        _require_device(t, n)
        if t.dtype != torch.bfloat16:
            raise RuntimeError(f"rms_norm: {n} must be bfloat16")
        if not t.is_contiguous():
            raise RuntimeError(f"rms_norm: {n} must be contiguous")
    H = x.shape[-1]
    if weight.numel() != H or out.shape != x.shape:
        raise RuntimeError("rms_norm: shape mismatch")
    T = x.numel() // H
    _lib.check(_lib.load().mcpu_rms_norm(out.data_ptr(), x.data_ptr(), weight.data_ptr(), T, H,
                                         float(eps), 1, _stream_handle(x.device)), "rms_norm")


def _check_bf16_2d(t: torch.Tensor, name: str) -> None:
    _require_device(t, name)
    if t.dtype != torch.bfloat16 or t.dim() != 2:
        raise RuntimeError(f"{name} must be a 2-D bfloat16 tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def mm_nt(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
          bias: torch.Tensor | None = None) -> torch.Tensor:
    """out = a @ b.T (+ bias), i.e. torch.mm(a, b.t()) for an nn.Linear weight
    b [N, K]; aten::mm / aten::addmm of the reference (csrc/aten/ops/mm.cpp)."""
    _check_bf16_2d(a, "a")
    _check_bf16_2d(b, "b")
    M, K = a.shape
    N, K2 = b.shape
    if K != K2:
        raise RuntimeError(f"mm: a.size(1) ({K}) must match b.size(1) ({K2})")
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    elif tuple(out.shape) != (M, N) or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise RuntimeError(f"mm: out must be a contiguous bfloat16 [{M}, {N}] tensor")
    lib = _lib.load()
    s = _stream_handle(a.device)
    if bias is None:
        _lib.check(lib.mcpu_mm(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, 1, s), "mm")
    else:
        if bias.numel() != N or bias.dtype != torch.bfloat16:
            raise RuntimeError("addmm: bias must be bfloat16 [N]")
        bias = bias.contiguous()
        _lib.check(lib.mcpu_addmm(bias.data_ptr(), a.data_ptr(), b.data_ptr(), out.data_ptr(),
                                  M, N, K, 1, s), "addmm")
    return out


def interleave_gate_up(w_gate_up: torch.Tensor, block: int = 128) -> torch.Tensor:
    """[gate; up] stacked rows [2I, K] -> the 128-row interleaved layout the
    fused gate/up GEMM reads (done once, when weights are loaded)."""
    two_i, K = w_gate_up.shape
    I = two_i // 2
    if two_i != 2 * I or I % block != 0:
        raise RuntimeError(f"interleave_gate_up: intermediate size {I} must be a multiple of {block}")
    return (w_gate_up.view(2, I // block, block, K).transpose(0, 1).reshape(two_i, K).contiguous())


def gemm_swiglu(x: torch.Tensor, w_gate_up_interleaved: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """out = silu(x @ Wg.T) * (x @ Wu.T) with the reference's bf16 roundings,
    one kernel (see interleave_gate_up for the weight layout)."""
    _check_bf16_2d(x, "x")
    _check_bf16_2d(w_gate_up_interleaved, "w_gate_up")
    M, K = x.shape
    two_i, K2 = w_gate_up_interleaved.shape
    if K != K2:
        raise RuntimeError("gemm_swiglu: K mismatch")
    I = two_i // 2
    if out is None:
        out = torch.empty(M, I, dtype=torch.bfloat16, device=x.device)
    _lib.check(_lib.load().mcpu_gemm_swiglu(x.data_ptr(), w_gate_up_interleaved.data_ptr(),
                                            out.data_ptr(), M, I, K, 1, _stream_handle(x.device)),
               "gemm_swiglu")
    return out


def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int,
                         expert_map: torch.Tensor | None = None, pad_sorted_ids: bool = False):
    """Per-expert token lists for the fused-MoE GEMMs, with the signature and
    outputs of vLLM's moe_align_block_size
    (vllm/model_executor/layers/fused_moe/moe_align_block_size.py:11-18):
    (sorted_token_ids, expert_ids, num_tokens_post_pad).  Runs are in
    ascending flat index; slots after the last run hold numel and blocks past
    it have expert -1."""
    import ctypes

    _require_device(topk_ids, "topk_ids")
    if expert_map is not None:
        raise NotImplementedError("moe_align_block_size: expert_map is not supported")
    ids = topk_ids.to(torch.int32).contiguous()
    numel = ids.numel()
    cap = min(numel + num_experts * (block_size - 1), numel * block_size)
    if pad_sorted_ids:
        cap = -(-cap // block_size) * block_size
    nblocks = -(-cap // block_size)
    dev = ids.device
    sorted_ids = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)[:cap]
    expert_ids = torch.empty(max(nblocks, 1), dtype=torch.int32, device=dev)[:nblocks]
    post_pad = torch.empty(1, dtype=torch.int32, device=dev)
    lib = _lib.load()
    ws = ctypes.c_uint64()
    _lib.check(lib.mcpu_moe_align_workspace_bytes(numel, num_experts, ctypes.byref(ws)), "moe_align_block_size")
    work = torch.empty(ws.value, dtype=torch.uint8, device=dev)
    _lib.check(lib.mcpu_moe_align_block_size(ids.data_ptr(), numel, num_experts, block_size, sorted_ids.data_ptr(),
                                             sorted_ids.numel(), expert_ids.data_ptr(), expert_ids.numel(),
                                             post_pad.data_ptr(), work.data_ptr(), ws.value, _stream_handle(dev)),
               "moe_align_block_size")
    return sorted_ids, expert_ids, post_pad


_DISPATCH_WS: dict = {}


def _dispatch_workspace(dev: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """Zero-filled workspace of grouped_topk_moe_align, one per (device,
    stream): each call leaves it ready for the next, so it is reused as is."""
    key = (dev.index, stream)
    ws = _DISPATCH_WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        _DISPATCH_WS[key] = ws
    return ws


def grouped_topk_moe_align(
    hidden_states: torch.Tensor,
    gating_output: torch.Tensor,
    topk: int,
    renormalize: bool,
    num_expert_group: int,
    topk_group: int,
    scoring_func: str = "softmax",
    routed_scaling_factor: float = 1.0,
    e_score_correction_bias: torch.Tensor | None = None,
    block_size: int = 64,
):
    """grouped_topk followed by moe_align_block_size on its ids, as vLLM's
    fused MoE runs them; one launch for DeepSeek-V3's router shape.  Returns
    (topk_weights, topk_ids, sorted_token_ids, expert_ids, num_tokens_post_pad),
    bit-identical to the two ops called one after the other."""
    import ctypes

    if hidden_states.size(0) != gating_output.size(0):
        raise AssertionError("Number of tokens mismatch")
    if scoring_func not in _SCORING:
        raise ValueError(f"Unsupported scoring function: {scoring_func}")
    _require_device(gating_output, "gating_output")
    if gating_output.dim() != 2 or gating_output.dtype not in _DTYPES:
        raise RuntimeError("grouped_topk_moe_align: gating_output must be a float32 or bfloat16 "
                           "[num_tokens, num_experts] tensor")
    g = gating_output.contiguous()
    T, E = g.shape
    bias = None
    if e_score_correction_bias is not None:
        _require_device(e_score_correction_bias, "e_score_correction_bias")
        if e_score_correction_bias.numel() != E:
            raise RuntimeError("grouped_topk: e_score_correction_bias must have num_experts elements")
        bias = e_score_correction_bias.to(torch.float32).contiguous()
    dev = g.device
    numel = T * topk
    cap = min(numel + E * (block_size - 1), numel * block_size)
    nblocks = -(-cap // block_size)
    w = torch.empty(T, topk, dtype=torch.float32, device=dev)
    ids = torch.empty(T, topk, dtype=torch.int32, device=dev)
    sorted_ids = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)[:cap]
    expert_ids = torch.empty(max(nblocks, 1), dtype=torch.int32, device=dev)[:nblocks]
    post_pad = torch.empty(1, dtype=torch.int32, device=dev)
    lib = _lib.load()
    nb = ctypes.c_uint64()
    _lib.check(lib.mcpu_grouped_topk_moe_align_workspace_bytes(T, E, topk, ctypes.byref(nb)),
               "grouped_topk_moe_align")
    stream = _stream_handle(dev)
    ws = _dispatch_workspace(dev, stream, nb.value)
    _lib.check(lib.mcpu_grouped_topk_moe_align(
        g.data_ptr(), _DTYPES[g.dtype], T, E, num_expert_group, topk_group, topk, int(bool(renormalize)),
        float(routed_scaling_factor), None if bias is None else bias.data_ptr(), _SCORING[scoring_func],
        w.data_ptr(), ids.data_ptr(), block_size, sorted_ids.data_ptr(), sorted_ids.numel(),
        expert_ids.data_ptr(), expert_ids.numel(), post_pad.data_ptr(), ws.data_ptr(), ws.numel(), stream),
        "grouped_topk_moe_align")
    return w, ids, sorted_ids, expert_ids, post_pad


def device_error(reset: bool = False) -> int:
    """1 if a kernel gave up on a bounded wait since the last reset."""
    import ctypes

    f = ctypes.c_int(0)
    _lib.check(_lib.load().mcpu_device_error(ctypes.byref(f), int(reset)), "device_error")
    return int(f.value)


def _elementwise(fn_name: str, x: torch.Tensor) -> torch.Tensor:
    _require_device(x, "x")
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise RuntimeError(f"{fn_name}: float32 or bfloat16 only")
    x = x.contiguous()
    out = torch.empty_like(x)
    fn = getattr(_lib.load(), "mcpu_" + fn_name)
    _lib.check(fn(out.data_ptr(), x.data_ptr(), x.numel(), _DTYPES[x.dtype], _stream_handle(x.device)), fn_name)
    return out


def sigmoid(x: torch.Tensor) -> torch.Tensor:
    """1 / (1 + exp(-x)) with exp correctly rounded: the reference's raw
    sigmoid loop (csrc/aten/ops/unary_out.cpp:46-49)."""
    return _elementwise("sigmoid", x)


def silu(x: torch.Tensor) -> torch.Tensor:
    """x / (1 + exp(-x)) with exp correctly rounded (unary_out.cpp:50-51)."""
    return _elementwise("silu", x)
