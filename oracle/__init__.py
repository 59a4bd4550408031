"""CPU oracle for the torch_mcpu device hot path.

TEST INFRASTRUCTURE ONLY.  tests/, the smoke check in __graft_entry__.py and
the CPU legs of bench.py import this package as the checker.  The product
package (torch_mcpu_b200) never imports it.

The arithmetic lives in oracle.c (built by oracle/Makefile into
oracle/build/liboracle.so); this module wraps it with numpy arrays and adds the
numpy restatement of the tensor-parallel MLP of the reference's
example/01_mlp_tp4/run.py:35-56,106-126 in the gated (SwiGLU) form the
benchmark configurations use.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "build", "liboracle.so")
_lib = None

EXP_GLIBC = 0
EXP_CR = 1
SOFTMAX = 0
SIGMOID = 1


def build() -> str:
    """Compile oracle.c with the committed Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
        os.path.join(_HERE, "oracle.c")
    ):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    P = ctypes.c_void_p
    lib.oracle_grouped_topk.argtypes = [
        P, ctypes.c_int, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_float, P, ctypes.c_int, ctypes.c_int,
        P, P, P, P, ctypes.c_int,
    ]
    lib.oracle_grouped_topk.restype = ctypes.c_int
    lib.oracle_silu_and_mul_bf16.argtypes = [P, ctypes.c_int64, ctypes.c_int64, P, ctypes.c_int, ctypes.c_int]
    lib.oracle_silu_and_mul_bf16.restype = ctypes.c_int
    lib.oracle_rms_norm_bf16.argtypes = [P, P, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, P, ctypes.c_int]
    lib.oracle_rms_norm_bf16.restype = ctypes.c_int
    lib.oracle_sigmoid_f32.argtypes = [P, ctypes.c_int64, P, ctypes.c_int]
    lib.oracle_sigmoid_f32.restype = None
    lib.oracle_silu_raw_bf16.argtypes = [P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, P, ctypes.c_int]
    lib.oracle_silu_raw_bf16.restype = None
    _lib = lib
    return lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def grouped_topk(
    gating: np.ndarray,
    topk: int,
    renormalize: bool,
    num_expert_group: int,
    topk_group: int,
    scoring_func: str = "softmax",
    routed_scaling_factor: float = 1.0,
    e_score_correction_bias: np.ndarray | None = None,
    exp_mode: int = EXP_GLIBC,
    nthreads: int = 0,
):
    """Oracle grouped_topk (tests/test_grouped_topk_compile.py:15-66).

    gating: [T, E] float32, or uint16 holding bf16 bits.
    Returns (weights f32 [T, K], ids i32 [T, K], tie_rows bool [T], gaps f32 [T]).
    """
    lib = _load()
    g = np.ascontiguousarray(gating)
    if g.dtype == np.float32:
        dt = 0
    elif g.dtype == np.uint16:
        dt = 1
    else:
        raise TypeError(f"gating must be float32 or bf16 bits (uint16), got {g.dtype}")
    T, E = g.shape
    bias = None
    if e_score_correction_bias is not None:
        bias = np.ascontiguousarray(e_score_correction_bias, dtype=np.float32)
        assert bias.shape == (E,)
    w = np.empty((T, topk), np.float32)
    ids = np.empty((T, topk), np.int32)
    ties = np.empty((T,), np.uint8)
    gaps = np.empty((T,), np.float32)
    scoring = {"softmax": SOFTMAX, "sigmoid": SIGMOID}[scoring_func]
    rc = lib.oracle_grouped_topk(
        _ptr(g), dt, T, E, num_expert_group, topk_group, topk, int(bool(renormalize)),
        float(routed_scaling_factor), _ptr(bias), scoring, exp_mode,
        _ptr(w), _ptr(ids), _ptr(ties), _ptr(gaps), nthreads,
    )
    if rc != 0:
        raise ValueError(f"oracle_grouped_topk rejected its arguments (code {rc})")
    return w, ids, ties.astype(bool), gaps


def silu_and_mul_bf16(x_bits: np.ndarray, exp_mode: int = EXP_GLIBC, nthreads: int = 0) -> np.ndarray:
    """x_bits: uint16 [T, 2d] bf16 bits -> uint16 [T, d]."""
    lib = _load()
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    T, two_d = x.shape
    d = two_d // 2
    out = np.empty((T, d), np.uint16)
    rc = lib.oracle_silu_and_mul_bf16(_ptr(x), T, d, _ptr(out), exp_mode, nthreads)
    assert rc == 0
    return out


def rms_norm_bf16(x_bits: np.ndarray, w_bits: np.ndarray, eps: float, nthreads: int = 0) -> np.ndarray:
    lib = _load()
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    T, H = x.shape
    out = np.empty((T, H), np.uint16)
    rc = lib.oracle_rms_norm_bf16(_ptr(x), _ptr(w), T, H, float(eps), _ptr(out), nthreads)
    assert rc == 0
    return out


def sigmoid_f32(x: np.ndarray, exp_mode: int = EXP_GLIBC) -> np.ndarray:
    lib = _load()
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib.oracle_sigmoid_f32(_ptr(x), x.size, _ptr(out), exp_mode)
    return out


def silu_raw_bf16(x_bits: np.ndarray, d: int, exp_mode: int = EXP_GLIBC) -> np.ndarray:
    """The reference's single-threaded raw silu loop on the first d columns
    of x (bf16 bits [T, pitch]) -> bf16 bits [T, d]."""
    lib = _load()
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    T, pitch = x.shape
    out = np.empty((T, d), np.uint16)
    lib.oracle_silu_raw_bf16(_ptr(x), T, d, pitch, _ptr(out), exp_mode)
    return out


# ---------------------------------------------------------------- bf16 helpers
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even, as c10::BFloat16 does for finite values."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    if nan.any():
        r[nan] = 0x7FC0
    return r


# ---------------------------------------------------------------- MLP
def gemm_bf16(a_bits: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
    """C = A @ W^T with bf16 operands, fp64 accumulation, bf16 result
    (csrc/aten/ops/mm.cpp:13-43 runs at::mm_out on CPU: bf16 in, fp32
    accumulation, bf16 out)."""
    a = bf16_bits_to_f32(a_bits).astype(np.float64)
    w = bf16_bits_to_f32(w_bits).astype(np.float64)
    return f32_to_bf16_bits((a @ w.T).astype(np.float32))


def tp_mlp_bf16(
    x_bits: np.ndarray,
    w_gate_up_shards: list[np.ndarray],
    w_down_shards: list[np.ndarray],
    rms_weight_bits: np.ndarray | None = None,
    eps: float = 1e-6,
    exp_mode: int = EXP_GLIBC,
) -> np.ndarray:
    """Tensor-parallel gated MLP, one shard per rank, then the SUM all-reduce
    (example/01_mlp_tp4/run.py:50-56 forward, 106-113 step).

    Each rank: h = x (optionally rms_norm'd) ; gu = h @ Wgu_r^T (bf16) ;
    a = silu(gu[:, :I_r]) * gu[:, I_r:] (bf16) ; y_r = a @ Wd_r^T (bf16).
    Output: bf16(sum_r y_r) with the sum in fp32.
    """
    h = x_bits
    if rms_weight_bits is not None:
        h = rms_norm_bf16(x_bits, rms_weight_bits, eps)
    acc = None
    for wgu, wd in zip(w_gate_up_shards, w_down_shards):
        gu = gemm_bf16(h, wgu)
        a = silu_and_mul_bf16(gu, exp_mode)
        y = bf16_bits_to_f32(gemm_bf16(a, wd))
        acc = y if acc is None else acc + y
    return f32_to_bf16_bits(acc)


# ---------------------------------------------------------------- MoE dispatch
def moe_align_block_size(topk_ids: np.ndarray, num_experts: int, block_size: int,
                         sorted_capacity: int | None = None):
    """Per-expert token lists after the router, with the contract of vLLM's
    moe_align_block_size (vllm/_custom_ops.py:2247-2264, documented with a
    worked example in vllm/model_executor/layers/fused_moe/
    moe_align_block_size.py:19-73): the flat indices of topk_ids grouped by
    expert, each expert's run padded with numel to a multiple of block_size.
    Runs are in ascending flat index (a stable counting sort); slots after the
    last run hold numel; expert_ids is -1 past the last run; entries outside
    [0, num_experts) are left out.

    Returns (sorted_token_ids int32 [capacity], expert_ids int32
    [ceil(capacity / block_size)], num_tokens_post_pad int)."""
    ids = np.asarray(topk_ids, dtype=np.int64).reshape(-1)
    numel = ids.size
    if sorted_capacity is None:
        sorted_capacity = min(numel + num_experts * (block_size - 1), numel * block_size)
    valid = (ids >= 0) & (ids < num_experts)
    counts = np.bincount(ids[valid], minlength=num_experts)
    padded = (counts + block_size - 1) // block_size * block_size
    start = np.concatenate([[0], np.cumsum(padded)])
    out = np.full(sorted_capacity, numel, dtype=np.int32)
    order = np.nonzero(valid)[0]
    order = order[np.argsort(ids[order], kind="stable")]
    pos = 0
    for e in range(num_experts):
        c = counts[e]
        out[start[e]:start[e] + c] = order[pos:pos + c]
        pos += c
    nblocks = -(-sorted_capacity // block_size)
    eids = np.full(nblocks, -1, dtype=np.int32)
    for e in range(num_experts):
        eids[start[e] // block_size:start[e + 1] // block_size] = e
    return out, eids, int(start[-1])


# ---------------------------------------------------------------- sampler
def _row_max_ref(row: np.ndarray) -> np.float32:
    # a running `x > max` from -inf: NaN never becomes the maximum
    finite = row[~np.isnan(row)]
    return np.float32(finite.max()) if finite.size else np.float32(-np.inf)


def vllm_min_p(logits: np.ndarray, idx: np.ndarray, min_p: np.ndarray, vocab: int) -> np.ndarray:
    """min_p.cpp:13-58 of the reference: per token row, with p =
    min_p[idx[t]], p == 0 leaves the row; else every entry (as fp32) below
    rowmax + logf(p) becomes -inf.  logits: fp32 values of the rows (exact
    for fp16/bf16 inputs); returns the new fp32 values."""
    out = np.array(logits, dtype=np.float32, copy=True)
    for t in range(out.shape[0]):
        p = np.float32(min_p[idx[t]])
        if p == 0:
            continue
        row = out[t, :vocab]
        with np.errstate(invalid="ignore", divide="ignore"):
            thr = np.float32(_row_max_ref(row) + np.float32(np.log(np.float64(p))))
            row[row < thr] = -np.inf
    return out


def vllm_topk_log_softmax(logits: np.ndarray, ids: np.ndarray, vocab: int) -> np.ndarray:
    """logprob.cpp:15-69: out[r, k] = logits[r, id] - lse, lse = max +
    (float)log(sum exp((double)(x - max))), id clamped to [0, vocab)."""
    lg = np.asarray(logits, dtype=np.float32)
    out = np.empty(ids.shape, dtype=np.float32)
    for r in range(lg.shape[0]):
        row = lg[r, :vocab]
        m = _row_max_ref(row)
        with np.errstate(invalid="ignore", over="ignore"):
            se = np.exp((row - m).astype(np.float64)).sum()
            lse = np.float32(m + np.float32(np.log(se)))
        for k in range(ids.shape[1]):
            i = min(max(int(ids[r, k]), 0), vocab - 1)
            out[r, k] = np.float32(row[i] - lse)
    return out


def vllm_ranks(logits: np.ndarray, token_ids: np.ndarray, vocab: int) -> np.ndarray:
    """logprob.cpp:123-149: out[r] = number of entries >= logits[r, token]."""
    lg = np.asarray(logits, dtype=np.float32)
    return np.array([int((lg[r, :vocab] >= lg[r, int(token_ids[r])]).sum()) for r in range(lg.shape[0])],
                    dtype=np.int64)


def vllm_penalties(logits: np.ndarray, idx: np.ndarray, token_ids: np.ndarray, local_pos: np.ndarray,
                   rep: np.ndarray, freq: np.ndarray, pres: np.ndarray, prompt_bin_mask: np.ndarray,
                   output_bin_counts: np.ndarray, vocab: int, max_spec_len: int) -> np.ndarray:
    """penalties.cpp:14-84: repetition / frequency / presence penalties of
    each token row, returned as new fp32 logits.  count[v] = output count of
    the row's request plus the row's draft tokens token_ids[t-pos+1 .. t]
    equal to v (pos = local_pos[t] > 0 and max_spec_len > 0); where rep != 1
    and v is in the prompt bit mask or count > 0: l / rep for l > 0, else
    l * rep; then l - freq * count, l - pres * [count > 0], each an fp32
    operation."""
    lg = np.array(logits, dtype=np.float32, copy=True)
    v = np.arange(vocab)
    for t in range(lg.shape[0]):
        q = int(idx[t])
        rp, fp, pp = np.float32(rep[q]), np.float32(freq[q]), np.float32(pres[q])
        if rp == 1 and fp == 0 and pp == 0:
            continue
        cnt = np.array(output_bin_counts[q, :vocab], dtype=np.int64)
        pos = int(local_pos[t])
        if pos > 0 and max_spec_len > 0:
            for prev in range(pos):
                d = int(token_ids[t - pos + prev + 1])
                if 0 <= d < vocab:
                    cnt[d] += 1
        out = cnt > 0
        x = lg[t, :vocab].copy()
        if rp != 1:
            words = np.asarray(prompt_bin_mask[q], dtype=np.int32).view(np.uint32)[v >> 5]
            hit = ((words >> (v & 31).astype(np.uint32)) & 1).astype(bool) | out
            x = np.where(hit, np.where(x > 0, x / rp, x * rp), x).astype(np.float32)
        x = (x - fp * cnt.astype(np.float32)).astype(np.float32)
        x = (x - pp * out.astype(np.float32)).astype(np.float32)
        lg[t, :vocab] = x
    return lg


def vllm_bincount(idx: np.ndarray, all_token_ids: np.ndarray, prompt_len: np.ndarray, prefill_len: np.ndarray,
                  prompt_bin_mask: np.ndarray, output_bin_counts: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """penalties.cpp:187-246: for each listed request q, bit tok of the prompt
    mask row q for the first prompt_len[q] tokens, +1 in the output counts
    row q for tokens prompt_len[q] .. prefill_len[q]; tokens outside the mask
    or the vocabulary are skipped.  Accumulates into copies of the inputs."""
    pbm = np.array(prompt_bin_mask, dtype=np.int32, copy=True)
    obc = np.array(output_bin_counts, dtype=np.int32, copy=True)
    pu = pbm.view(np.uint32)
    cols, vocab = pbm.shape[1], obc.shape[1]
    for q in np.asarray(idx, dtype=np.int64):
        p, f = int(prompt_len[q]), int(prefill_len[q])
        pt = np.asarray(all_token_ids[q, :p], dtype=np.int64)
        pt = pt[(pt >= 0) & (pt // 32 < cols)]
        np.bitwise_or.at(pu[q], pt // 32, (np.uint32(1) << (pt % 32).astype(np.uint32)))
        ot = np.asarray(all_token_ids[q, p:f], dtype=np.int64)
        np.add.at(obc[q], ot[(ot >= 0) & (ot < vocab)], 1)
    return pbm, obc


def vllm_bias(logits: np.ndarray, vocab: int, idx: np.ndarray, num_allowed: np.ndarray, allowed: np.ndarray,
              num_bias: np.ndarray, bias_ids: np.ndarray, bias: np.ndarray, pos: np.ndarray,
              min_lens: np.ndarray, num_stop: np.ndarray, stop_ids: np.ndarray,
              rnd=lambda v: np.float32(v)) -> np.ndarray:
    """logit_bias.cpp:15-96, per token row in order: (1) with allowed tokens,
    keep the values of the first min(n, 512) allowed ids (clamped into the
    vocabulary) and set the rest of the row to -inf; (2) add each bias to its
    id in list order, rounding to the logits dtype after each add (`rnd`);
    (3) while pos < min_len, set the stop ids to -inf.  Values are fp32
    copies of the logits dtype; returns new logits."""
    lg = np.array(logits, dtype=np.float32, copy=True)
    for t in range(lg.shape[0]):
        q = int(idx[t])
        row = lg[t]
        na = int(num_allowed[q])
        if na > 0:
            ids = np.clip(np.asarray(allowed[q, :min(na, 512)], dtype=np.int64), 0, vocab - 1)
            keep = row[ids].copy()
            row[:vocab] = -np.inf
            row[ids] = keep
        for k in range(int(num_bias[q])):
            i = int(bias_ids[q, k])
            if 0 <= i < vocab:
                row[i] = rnd(np.float32(row[i]) + np.float32(bias[q, k]))
        if int(num_stop[q]) > 0 and int(pos[t]) < int(min_lens[q]):
            for k in range(int(num_stop[q])):
                i = int(stop_ids[q, k])
                if 0 <= i < vocab:
                    row[i] = -np.inf
    return lg


def vllm_bad_words(logits: np.ndarray, idx: np.ndarray, bw_ids: np.ndarray, bw_off: np.ndarray, n_bw: np.ndarray,
                   all_token_ids: np.ndarray, prompt_len: np.ndarray, total_len: np.ndarray,
                   input_ids: np.ndarray, local_pos: np.ndarray) -> np.ndarray:
    """bad_words.cpp:13-82: for token row t (request q, local position pos),
    every bad word ids[off[w] .. off[w+1]) whose prefix equals the last
    tokens of q's output (all_token_ids[q, prompt_len .. total_len)) followed
    by the drafts input_ids[t-pos .. t) bans its last id (-inf).  Returns
    new logits; the vocabulary is the row width."""
    lg = np.array(logits, dtype=np.float32, copy=True)
    vocab = lg.shape[1]
    for t in range(lg.shape[0]):
        q = int(idx[t])
        nw = int(n_bw[q])
        if nw == 0:
            continue
        pos = int(local_pos[t])
        pl, tl = int(prompt_len[q]), int(total_len[q])
        out_len = tl - pl
        eff = out_len + pos
        seq = list(all_token_ids[q, pl:tl]) + list(input_ids[t - pos:t])
        for w in range(nw):
            start, end = int(bw_off[q, w]), int(bw_off[q, w + 1])
            prefix = end - start - 1
            if prefix > eff:
                continue
            want = [int(v) for v in bw_ids[q, start:start + max(prefix, 0)]]
            have = [int(v) for v in seq[eff - max(prefix, 0):eff]] if prefix > 0 else []
            last = int(bw_ids[q, end - 1])
            if want == have and 0 <= last < vocab:
                lg[t, last] = -np.inf
    return lg
