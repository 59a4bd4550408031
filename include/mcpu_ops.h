/*
 * Hot-path op entry points of the mcpu device on B200 (sm_100a): a C-ABI of
 * plain pointers, sizes and a stream.  Every pointer named "device" is HBM
 * (orMalloc / cudaMalloc / a torch CUDA tensor's data_ptr); every call is
 * asynchronous on `stream` like the reference's ops, which return after
 * enqueueing on the current mcpu stream (docs/kernel_launch_migration.md,
 * "Migration checkpoints").
 *
 * Error behaviour: argument problems return orErrorInvalidValue and launch
 * failures orErrorUnknown, with the message in mcpuGetLastErrorString();
 * the Python layer raises RuntimeError with it, where the reference raises
 * c10::Error from TORCH_CHECK.  There is no CPU fallback: with no usable
 * device the call fails.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "openreg.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef enum mcpuDtype {
  MCPU_FLOAT32 = 0,
  MCPU_BFLOAT16 = 1,
  MCPU_FLOAT16 = 2,
  MCPU_INT32 = 3,
  MCPU_INT64 = 4,
  MCPU_UINT8 = 5,
  MCPU_BOOL = 6,
  MCPU_FLOAT64 = 7,
  MCPU_INT8 = 8,
  MCPU_INT16 = 9
} mcpuDtype;

typedef enum mcpuScoring {
  MCPU_SCORING_SOFTMAX = 0,
  MCPU_SCORING_SIGMOID = 1
} mcpuScoring;

/* Text of the last error raised on this host thread ("" if none). */
OPENREG_EXPORT const char* mcpuGetLastErrorString(void);

/*
 * Grouped top-k MoE router, one fused kernel.
 *
 * Replaces the aten chain of copied_grouped_topk
 * (tests/test_grouped_topk_compile.py:15-66), which on the reference runs as
 * sigmoid (csrc/aten/ops/unary_out.cpp:415-430) or _softmax
 * (csrc/aten/ops/softmax_random_argmax.cpp:57-82), add
 * (binary_out.cpp:259), three topk (topk.cpp:10-40), sum/max
 * (reduction_scatter.cpp:116-150, 461-495), the scatter/masked_fill mask
 * (unary_out.cpp:684-700; scatter.value_out falls back to CPU), gather
 * (gather.cpp:10-31), div and mul (binary_out.cpp:307, 544).
 *
 * gating        device, [num_tokens, num_experts] row-major, fp32 or bf16
 * bias          device fp32 [num_experts] or NULL (e_score_correction_bias)
 * topk_weights  device fp32 [num_tokens, topk]
 * topk_ids      device int32 [num_tokens, topk]
 *
 * Constraints: num_experts % num_expert_group == 0, num_expert_group a power
 * of two <= 32, group size <= 64 (>= 2 with a bias), topk <= 16,
 * topk <= topk_group * group size, num_experts <= 1024.
 *
 * Semantics: experts are ranked by the biased score (score + bias) when a
 * bias is given, else by the logit (order-equivalent to softmax/sigmoid);
 * ties go to the lower index (group or expert).  Outputs are ordered by rank.
 * Sigmoid scores equal 1/(1 + e^-x) with e^-x correctly rounded to fp32.
 */
OPENREG_EXPORT orError_t mcpu_grouped_topk(
    const void* gating, int gating_dtype, int64_t num_tokens, int num_experts,
    int num_expert_group, int topk_group, int topk, int renormalize,
    float routed_scaling_factor, const float* bias, int scoring_func,
    float* topk_weights, int32_t* topk_ids, orStream_t stream);

/* Number of rows the router resolved on its exact (near-tie) path since the
 * last reset, summed over all launches on the current device. */
OPENREG_EXPORT orError_t mcpu_grouped_topk_exact_rows(
    unsigned long long* count, int reset);

/*
 * grouped_topk_moe_align: the router followed by the expert dispatch, i.e.
 * mcpu_grouped_topk (arguments and outputs as above) and then
 * mcpu_moe_align_block_size on its topk_ids (numel = num_tokens * topk,
 * num_experts experts; block_size and the last five outputs as there) --
 * vLLM's fused-MoE sequence grouped_topk -> moe_align_block_size
 * (vllm/model_executor/layers/fused_moe/moe_align_block_size.py:19-73).
 * Results are bit-identical to the two calls.
 *
 * For DeepSeek-V3's router (fp32 logits, 256 experts in 8 groups,
 * topk_group 4, topk 8, sigmoid + bias) it is ONE cooperative launch: each
 * CTA routes a contiguous token range, counts its ids per expert, sorts
 * them by expert in shared memory, and after one grid-wide barrier (bounded:
 * a wait that runs out after 2 s sets mcpu_device_error) copies them to
 * their places.  Other configurations, or more than 65535 ids per SM, run
 * the router and the dispatch's two launches.
 *
 * workspace: device memory of
 * mcpu_grouped_topk_moe_align_workspace_bytes(num_tokens, num_experts, topk)
 * bytes (sized for the current device), 16-byte aligned and zero-filled
 * before its first call (e.g. one cudaMemset when it is allocated).  Each
 * call leaves it ready for the next, so one workspace serves any number of
 * calls ordered on one stream.  After a device error, zero-fill it again.
 * No counterpart in the reference (it runs the router's aten chain and has
 * no dispatch op).
 */
OPENREG_EXPORT orError_t mcpu_grouped_topk_moe_align(
    const void* gating, int gating_dtype, int64_t num_tokens, int num_experts, int num_expert_group,
    int topk_group, int topk, int renormalize, float routed_scaling_factor, const float* bias,
    int scoring_func, float* topk_weights, int32_t* topk_ids, int block_size, int32_t* sorted_token_ids,
    int64_t sorted_capacity, int32_t* expert_ids, int64_t expert_ids_capacity, int32_t* num_tokens_post_pad,
    void* workspace, uint64_t workspace_bytes, orStream_t stream);

OPENREG_EXPORT orError_t mcpu_grouped_topk_moe_align_workspace_bytes(int64_t num_tokens, int num_experts,
                                                                     int topk, uint64_t* bytes);

/*
 * silu_and_mul: out[t, j] = silu(x[t, j]) * x[t, d + j] for x [T, 2d],
 * out [T, d], both contiguous bf16 on the device.
 *
 * Replaces vLLM's SiluAndMul.forward_native
 * (vllm/model_executor/layers/activation.py:135-139) as the reference runs
 * it: the raw silu loop x / (1.0f + std::exp(-x)) rounded to bf16
 * (csrc/aten/ops/unary_out.cpp:50-51, silu_out 456-470), then aten mul
 * (csrc/aten/ops/binary_out.cpp:544-560) rounded to bf16.  Schema of the
 * matching custom op: mcpu::silu_and_mul(Tensor(a!) out, Tensor x) -> ().
 */
OPENREG_EXPORT orError_t mcpu_silu_and_mul(void* out, const void* x, int64_t num_tokens,
                                           int64_t d, int dtype, orStream_t stream);

/*
 * rms_norm: out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * weight) per row of
 * x [T, H] (bf16), weight [H] (bf16), out [T, H] (bf16).
 *
 * Replaces vLLM's rms_norm native implementation
 * (vllm/ir/ops/layernorm.py:14-21), which the reference runs as pow and
 * rsqrt (CPU fallback), mean (csrc/aten/ops/reduction_scatter.cpp:248-285),
 * add and mul (binary_out.cpp).  Schema of the matching custom op:
 * mcpu::rms_norm(Tensor(a!) out, Tensor x, Tensor weight, float eps) -> ().
 */
OPENREG_EXPORT orError_t mcpu_rms_norm(void* out, const void* x, const void* weight,
                                       int64_t num_tokens, int64_t hidden, float eps,
                                       int dtype, orStream_t stream);

/*
 * mm: out[M, N] = a[M, K] . b[N, K]^T in bf16 with fp32 accumulation on the
 * tcgen05 tensor cores (TMA-fed shared-memory tiles, TMEM accumulators).
 * a, b, out contiguous row-major on the device, 16-byte aligned, K and N
 * multiples of 8 (the TMA stride rule).  b is the weight as stored by
 * nn.Linear, so this is torch.mm(a, b.t()).
 *
 * Replaces aten::mm / mm.out (csrc/aten/ops/mm.cpp:13-51), which calls
 * at::mm_out on host views of the operands.
 */
OPENREG_EXPORT orError_t mcpu_mm(const void* a, const void* b, void* out, int64_t M, int64_t N,
                                 int64_t K, int dtype, orStream_t stream);

/*
 * addmm: out = bf16(a . b^T + bias) with bias [N] bf16 added to the fp32
 * accumulator (one rounding).  Replaces aten::addmm / addmm.out
 * (csrc/aten/ops/mm.cpp:53-110).
 */
OPENREG_EXPORT orError_t mcpu_addmm(const void* bias, const void* a, const void* b, void* out,
                                    int64_t M, int64_t N, int64_t K, int dtype,
                                    orStream_t stream);

/*
 * gemm_swiglu: the gated MLP's gate/up projection with silu_and_mul fused
 * into the epilogue: out[M, I] = bf16(bf16(silu(bf16(x.Wg^T))) * bf16(x.Wu^T)),
 * i.e. exactly mm followed by mcpu_silu_and_mul, without writing the [M, 2I]
 * intermediate.  w_gate_up [2I, K] holds the gate and up rows interleaved in
 * blocks of 128: rows [256j, 256j+128) = Wg[128j .. 128j+128),
 * rows [256j+128, 256j+256) = Wu[128j .. 128j+128); I % 128 == 0.
 * Replaces the mm -> silu -> mul chain of the reference's TP MLP
 * (example/01_mlp_tp4/run.py:50-56) in its SwiGLU form.
 */
OPENREG_EXPORT orError_t mcpu_gemm_swiglu(const void* x, const void* w_gate_up, void* out,
                                          int64_t M, int64_t I, int64_t K, int dtype,
                                          orStream_t stream);

/*
 * Symmetric windows: one device buffer of the same size on every rank of a
 * tensor-parallel group (one process per GPU of one box), each rank mapping
 * all of them through CUDA IPC so kernels read and write peers' buffers over
 * NVLink.  The reference has no counterpart: its ProcessGroup stages tensors
 * through host memory (torch_mcpu/csrc/Distributed.cpp:281-354).
 *
 * symm_alloc: cudaMalloc of `bytes`, zero-filled (synchronously), and its
 * 64-byte IPC handle.  symm_open: maps another rank's handle into this
 * process (peer access enabled on first use).  symm_close undoes symm_open,
 * symm_free undoes symm_alloc.  symm_clear zeroes `bytes` at `ptr` on
 * `stream` (used to reset a window's counters after a failed call).
 */
#define MCPU_SYMM_MAX_RANKS 8
#define MCPU_SYMM_HANDLE_BYTES 64

typedef struct mcpuSymmWindow {
  int32_t rank;                         /* this process's rank, 0 <= rank < world */
  int32_t world;                        /* ranks in the group, 1..MCPU_SYMM_MAX_RANKS */
  uint64_t bytes;                       /* size of every rank's window */
  void* base[MCPU_SYMM_MAX_RANKS];      /* window of rank r as mapped in this process */
} mcpuSymmWindow;

OPENREG_EXPORT orError_t mcpu_symm_alloc(uint64_t bytes, void** ptr, uint8_t* handle);
OPENREG_EXPORT orError_t mcpu_symm_open(const uint8_t* handle, void** ptr);
OPENREG_EXPORT orError_t mcpu_symm_close(void* ptr);
OPENREG_EXPORT orError_t mcpu_symm_free(void* ptr);
OPENREG_EXPORT orError_t mcpu_symm_clear(void* ptr, uint64_t bytes, orStream_t stream);

/*
 * mm_allreduce: the row-parallel down projection of the TP MLP and the SUM
 * all-reduce of its partial outputs in one kernel, i.e.
 *     out = sum over ranks r of bf16(a_r . b_r^T)     (every rank gets out)
 * with a [M, K] and b [N, K] this rank's shards (bf16, as for mcpu_mm),
 * N % 256 == 0, K > 0.  Replaces mm (csrc/aten/ops/mm.cpp:13-51) followed
 * by McpuBackend::allreduce (torch_mcpu/csrc/Distributed.cpp:403-413), the
 * pair example/01_mlp_tp4/run.py:106-113 runs per step.
 *
 * Each rank's tensor-core epilogue sends every 32-row slice of its bf16
 * partial straight into the window of the slice's owner rank; the owner
 * sums the `world` partials in fp32 in rank order, rounds once to bf16 and
 * writes the result into every rank's window.  All ranks therefore hold the
 * same bits.  *out receives this rank's result: M x N bf16, row-major,
 * inside its own window; it stays valid until the next mm_allreduce on the
 * window.  The window must hold mcpu_mm_allreduce_window_bytes(M, N, world)
 * bytes; every rank calls with the same M, N, K.
 *
 * One cooperative launch per call (all its blocks resident on the GPU);
 * waits on other ranks give up after 2 s and set mcpu_device_error, after
 * which the window's counters must be cleared on every rank (symm_clear of
 * the first mcpu_mm_allreduce_control_bytes bytes) before it is used again.
 * Calls on one window must be ordered on one stream per rank.
 */
OPENREG_EXPORT orError_t mcpu_mm_allreduce(const void* a, const void* b, int64_t M, int64_t N,
                                           int64_t K, int dtype, const mcpuSymmWindow* window,
                                           void** out, orStream_t stream);

/* Window size mm_allreduce needs for an M x N output over `world` ranks. */
OPENREG_EXPORT orError_t mcpu_mm_allreduce_window_bytes(int64_t M, int64_t N, int world,
                                                        uint64_t* bytes);

/* Leading bytes of a window of `bytes` that hold mm_allreduce's counters
 * (zero whenever no call is in flight). */
OPENREG_EXPORT orError_t mcpu_mm_allreduce_control_bytes(uint64_t bytes, int world,
                                                         uint64_t* control_bytes);

/*
 * moe_align_block_size: MoE expert dispatch after the router, with the
 * contract of vLLM's op of that name (vllm/_custom_ops.py:2247-2264): the
 * numel entries of topk_ids (int32 [T, topk] flattened; expert indices in
 * [0, num_experts), num_experts <= 1024) grouped by expert into
 * sorted_token_ids, each expert's run in ascending flat index and padded
 * with the value numel to a multiple of block_size; every slot after the
 * last run also holds numel.  expert_ids[b] is the expert of slots
 * [b*block_size, (b+1)*block_size), -1 past the last run;
 * *num_tokens_post_pad (device int32) the slots the runs fill.
 * sorted_capacity >= min(numel + num_experts*(block_size-1), numel*block_size),
 * expert_ids_capacity >= ceil(that / block_size).  workspace: device memory
 * of mcpu_moe_align_workspace_bytes(numel, num_experts) bytes, no initial
 * content needed.  Entries outside [0, num_experts) are left out and set
 * mcpu_device_error.  The reference has no such op: it would assemble the
 * lists from scatter_add / index ops (csrc/aten/ops/reduction_scatter.cpp:
 * 517-555) on host views.
 */
OPENREG_EXPORT orError_t mcpu_moe_align_block_size(const int32_t* topk_ids, int64_t numel, int num_experts,
                                                   int block_size, int32_t* sorted_token_ids,
                                                   int64_t sorted_capacity, int32_t* expert_ids,
                                                   int64_t expert_ids_capacity, int32_t* num_tokens_post_pad,
                                                   void* workspace, uint64_t workspace_bytes,
                                                   orStream_t stream);

OPENREG_EXPORT orError_t mcpu_moe_align_workspace_bytes(int64_t numel, int num_experts, uint64_t* bytes);

/*
 * moe_align_block_size_static: the same dispatch, for callers that cannot
 * allocate device memory when they dispatch experts -- an inference engine
 * that reserved all free memory for its own pool at start-up, code that must
 * not stall on cudaMalloc's device-wide synchronisation while serving, or a
 * C caller with no device allocator.  No workspace argument: the count
 * matrix lives in a fixed 256 KiB array of this library's device memory
 * (65536 int32 counters, kept on every GPU that loads the library until the
 * process exits), so ceil(numel / 4096) * num_experts must be <= 65536 --
 * up to 1,048,576 entries with 256 experts; larger calls fail with
 * orErrorInvalidValue and a message naming the limit.  It allocates nothing
 * and calls no allocating routine.  The first call on each device looks up
 * the array's device address (cudaGetSymbolAddress) on the current device;
 * CUDA loads a library's device code lazily, so that first call is also the
 * moment the 256 KiB array is placed in the device's memory: make it before
 * the caller reserves its memory pool, and before any stream capture.  The
 * address is kept per device for the life of the process; after a reset of
 * the device's primary context, make a first call again in a fresh process.
 * All calls share the array: calls whose kernels overlap on the GPU race,
 * so order them on one stream.  No counterpart in the reference.
 */
OPENREG_EXPORT orError_t mcpu_moe_align_block_size_static(const int32_t* topk_ids, int64_t numel, int num_experts,
                                                          int block_size, int32_t* sorted_token_ids,
                                                          int64_t sorted_capacity, int32_t* expert_ids,
                                                          int64_t expert_ids_capacity,
                                                          int32_t* num_tokens_post_pad, orStream_t stream);

/*
 * The reference's stream test ops (csrc/aten/native/Extra.cpp:255-296,
 * schemas mcpu::stream_sleep_fill_, stream_sleep_copy_, first_element_int),
 * which make stream ordering observable:
 *   mcpu_stream_sleep_fill_i64  on `stream`: wait sleep_ms (0..60000) on the
 *     GPU's timer, then set the numel int64 values of x to `value`;
 *   mcpu_stream_sleep_copy_i64  the same wait, then copy src into dst;
 *   mcpu_read_i64_now           *out = *src (device memory), read at once
 *     on a private stream: it does not wait for work queued on other
 *     streams (the reference reads host memory directly).
 */
OPENREG_EXPORT orError_t mcpu_stream_sleep_fill_i64(int64_t* x, int64_t numel, int64_t value, int64_t sleep_ms,
                                                    orStream_t stream);
OPENREG_EXPORT orError_t mcpu_stream_sleep_copy_i64(int64_t* dst, const int64_t* src, int64_t numel,
                                                    int64_t sleep_ms, orStream_t stream);
OPENREG_EXPORT orError_t mcpu_read_i64_now(const int64_t* src, int64_t* out);

/*
 * vLLM sampler kernels of the decode path, the reference's own mcpu ops
 * (csrc/aten/vllm_kernels/min_p.cpp, logprob.cpp; schemas
 * mcpu::vllm_min_p_kernel, vllm_topk_log_softmax_kernel, vllm_ranks_kernel).
 * logits: [rows, logits_stride] on the device, float32 / float16 / bfloat16
 * (dtype code), the first vocab_size columns used; values compared as fp32.
 *
 * min_p (min_p.cpp:13-58): for each token row, min_p[expanded_idx_mapping[t]]
 *   = p; p == 0 leaves the row; else entries < rowmax + logf(p) become -inf,
 *   in place.
 * topk_log_softmax (logprob.cpp:15-69): output[r, k] (fp32, [batch, topk]) =
 *   logits[r, id] - (rowmax + log(sum exp(x - rowmax))), the sum in fp64, id =
 *   topk_ids[r, k] (int64, row stride topk_ids_stride) clamped to the vocab.
 * ranks (logprob.cpp:123-149): output[r] (int64) = number of entries >=
 *   logits[r, token_ids[r]]; a token id outside the vocab gives 0 and sets
 *   mcpu_device_error (the reference reads out of bounds).
 */
OPENREG_EXPORT orError_t mcpu_vllm_min_p(void* logits, int dtype, int64_t num_tokens, int64_t logits_stride,
                                         const int32_t* expanded_idx_mapping, const float* min_p,
                                         int64_t vocab_size, orStream_t stream);
OPENREG_EXPORT orError_t mcpu_vllm_topk_log_softmax(float* output, const void* logits, int dtype, int64_t batch,
                                                    int64_t logits_stride, const int64_t* topk_ids,
                                                    int64_t topk_ids_stride, int64_t topk, int64_t vocab_size,
                                                    orStream_t stream);
OPENREG_EXPORT orError_t mcpu_vllm_ranks(int64_t* output, const void* logits, int dtype, int64_t batch,
                                         int64_t logits_stride, const int64_t* token_ids, int64_t vocab_size,
                                         orStream_t stream);

/*
 * Penalties (penalties.cpp:14-84, mcpu::vllm_penalties_kernel): for token
 *   row t of logits, request q = expanded_idx_mapping[t] (rep, freq, pres =
 *   the three penalty arrays [max_num_reqs] at q; rows with 1, 0, 0 are left
 *   as they are), count[v] = output_bin_counts[q, v] plus, when
 *   expanded_local_pos[t] = pos > 0 and max_spec_len > 0, the number of
 *   token_ids[t-pos+1 .. t] equal to v.  Where rep != 1 and v is in the prompt
 *   (bit v of prompt_bin_mask row q, int32 words) or count > 0, l = l / rep
 *   for l > 0 else l * rep; then l -= freq * count and l -= pres * [count > 0],
 *   each operation rounded to fp32, the result to the logits dtype, in place.
 *   A request index out of range, or pos > t, leaves the row and sets
 *   mcpu_device_error (the reference reads out of bounds).
 * Bincount (penalties.cpp:187-246, mcpu::vllm_bincount_kernel): for each of
 *   the num_reqs requests q = expanded_idx_mapping[i], sets bit tok of
 *   prompt_bin_mask row q for the all_token_ids[q, 0 .. prompt_len[q]) and
 *   adds 1 to output_bin_counts[q, tok] for all_token_ids[q, prompt_len[q] ..
 *   prefill_len[q]); tokens outside [0, vocab) are skipped; the outputs are
 *   accumulated into (zero them first).  A request index out of range, or
 *   lengths outside [0, max_seq_len], set mcpu_device_error.
 */
OPENREG_EXPORT orError_t mcpu_vllm_penalties(void* logits, int dtype, int64_t num_tokens, int64_t logits_stride,
                                             const int32_t* expanded_idx_mapping, const int32_t* token_ids,
                                             const int32_t* expanded_local_pos, const float* repetition_penalty,
                                             const float* frequency_penalty, const float* presence_penalty,
                                             int64_t max_num_reqs, const int32_t* prompt_bin_mask,
                                             int64_t pbm_stride, const int32_t* output_bin_counts,
                                             int64_t obc_stride, int64_t vocab_size, int64_t max_spec_len,
                                             orStream_t stream);
OPENREG_EXPORT orError_t mcpu_vllm_bincount(const int32_t* expanded_idx_mapping, int64_t num_reqs,
                                            const int32_t* all_token_ids, int64_t tids_stride,
                                            int64_t max_seq_len, const int32_t* prompt_len,
                                            const int32_t* prefill_len, int64_t max_num_reqs,
                                            int32_t* prompt_bin_mask, int64_t packed_cols, int64_t pbm_stride,
                                            int32_t* output_bin_counts, int64_t vocab_size, int64_t obc_stride,
                                            orStream_t stream);

/*
 * Logit bias (logit_bias.cpp:15-96, mcpu::vllm_bias_kernel), per token row t
 *   with request q = expanded_idx_mapping[t], in this order: (1) when
 *   num_allowed[q] = n > 0, the first min(n, 512) ids of allowed row q
 *   (clamped into [0, vocab)) keep their values and every other entry of the
 *   row becomes -inf; (2) bias[q, k] is added to logit bias_ids[q, k] for
 *   k < num_bias[q] in list order, rounded to the logits dtype after each
 *   add, ids outside the vocab skipped; (3) when pos[t] (int64) <
 *   min_lens[q], the first num_stop[q] stop ids become -inf.  A request index
 *   out of range leaves the row, and a count above its list's width is
 *   clamped; both set mcpu_device_error.
 */
OPENREG_EXPORT orError_t mcpu_vllm_bias(void* logits, int dtype, int64_t num_tokens, int64_t logits_stride,
                                        int64_t vocab_size, const int32_t* expanded_idx_mapping,
                                        int64_t max_num_reqs, const int32_t* num_allowed, const int32_t* allowed,
                                        int64_t allowed_stride, int64_t allowed_cols, const int32_t* num_bias,
                                        const int32_t* bias_ids, int64_t bias_ids_stride, const float* bias,
                                        int64_t bias_stride, int64_t bias_cols, const int64_t* pos,
                                        const int32_t* min_lens, const int32_t* num_stop, const int32_t* stop_ids,
                                        int64_t stop_stride, int64_t stop_cols, orStream_t stream);

/*
 * Bad words (bad_words.cpp:13-82, mcpu::vllm_bad_words_kernel): for token row
 *   t with request q and local position pos, each of the num_bad_words[q]
 *   words w = bad_word_token_ids[q, off[w] .. off[w+1]) (off = row q of
 *   bad_word_offsets) whose prefix (all ids but the last) equals the last
 *   tokens of q's output all_token_ids[q, prompt_len[q] .. total_len[q])
 *   followed by the drafts input_ids[t-pos .. t) gets its last id set to
 *   -inf in the row.  Indexes that would leave their tensors set
 *   mcpu_device_error and skip the word or row.
 */
OPENREG_EXPORT orError_t mcpu_vllm_bad_words(void* logits, int dtype, int64_t num_tokens, int64_t logits_stride,
                                             int64_t vocab_size, const int32_t* expanded_idx_mapping,
                                             int64_t max_num_reqs, const int32_t* bad_word_token_ids,
                                             int64_t bw_ids_stride, int64_t bw_ids_cols,
                                             const int32_t* bad_word_offsets, int64_t bw_off_stride,
                                             int64_t bw_off_cols, const int32_t* num_bad_words,
                                             const int32_t* all_token_ids, int64_t token_ids_stride,
                                             int64_t max_seq_len, const int32_t* prompt_len,
                                             const int32_t* total_len, const int32_t* input_ids,
                                             const int32_t* expanded_local_pos, orStream_t stream);

/* *flag = 1 if a kernel on the current device (tensor-core GEMM, TMA-fed
 * router or bulk-copy-fed rms_norm) gave up on a bounded wait, or a gather /
 * scatter met an index out of range, since the last reset; that launch left
 * its output incomplete.  No counterpart in the reference, whose host
 * worker threads report hangs through orStreamSynchronize's timeout. */
OPENREG_EXPORT orError_t mcpu_device_error(int* flag, int reset);

/* Free and total device memory of `device` (cudaMemGetInfo).  Backs
 * torch.mcpu.mem_get_info (torch_mcpu/openreg/__init__.py:391-395 of the
 * reference, where it reports the simulated device's memory). */
OPENREG_EXPORT orError_t mcpu_mem_get_info(int device, size_t* free_bytes, size_t* total_bytes);

/* Bytes reserved by the stream-ordered pool behind orMallocAsync on `device`
 * (current and high-water mark).  Backs torch.mcpu.memory_reserved /
 * max_memory_reserved (reference: the caching allocator's reserved bytes). */
OPENREG_EXPORT orError_t mcpu_mem_pool_reserved(int device, uint64_t* current, uint64_t* peak);

/*
 * CUDA graphs of mcpu work (no counterpart in the reference, whose host
 * queue replays nothing): capture everything enqueued on `stream` (a created
 * stream, thread-local capture mode) into an executable graph, replay it on
 * a stream, destroy it.  Work captured must not allocate device memory
 * (preallocate outputs); a graph holding NCCL calls is destroyed before the
 * process group is.
 */
OPENREG_EXPORT orError_t mcpu_graph_capture_begin(orStream_t stream);
OPENREG_EXPORT orError_t mcpu_graph_capture_end(orStream_t stream, void** graph_exec);
OPENREG_EXPORT orError_t mcpu_graph_launch(void* graph_exec, orStream_t stream);
OPENREG_EXPORT orError_t mcpu_graph_destroy(void* graph_exec);

/*
 * Tensor plumbing of the mcpu device (all asynchronous on `stream`).
 *
 * mcpu_copy_strided: dst[i] = convert(src[i]) over an ndim <= 8 index space
 * with element strides (either side may be non-contiguous); dtype
 * conversion follows torch's rules (through fp32 for bf16/fp16, truncation
 * toward zero for float -> int, nonzero -> 1 for bool).  Replaces the
 * device-side cases of _copy_from (csrc/aten/native/Minimal.cpp:393-484).
 *
 * mcpu_fill: every element of a strided view set to one value.  Replaces
 * fill_ / zero_ (csrc/aten/ops/fill.cpp:12-44, unary_out.cpp:239-267).
 */
OPENREG_EXPORT orError_t mcpu_copy_strided(const void* src, int src_dtype, void* dst, int dst_dtype,
                                           int ndim, const int64_t* sizes,
                                           const int64_t* src_strides, const int64_t* dst_strides,
                                           orStream_t stream);
OPENREG_EXPORT orError_t mcpu_fill(void* dst, int dtype, int ndim, const int64_t* sizes,
                                   const int64_t* strides, double fvalue, int64_t ivalue,
                                   int value_is_float, orStream_t stream);

/*
 * Elementwise ops on contiguous buffers of n elements (fp32 or bf16):
 * sigmoid = 1 / (1 + exp(-x)), silu = x / (1 + exp(-x)) in fp32 with exp
 * correctly rounded (the raw loops of csrc/aten/ops/unary_out.cpp:46-51,
 * sigmoid_out 415-430, silu_out 456-470; bf16 results are rounded from the
 * fp32 value), mul = a * b rounded to the dtype (binary_out.cpp:544-560).
 */
OPENREG_EXPORT orError_t mcpu_sigmoid(void* out, const void* x, int64_t n, int dtype,
                                      orStream_t stream);
OPENREG_EXPORT orError_t mcpu_silu(void* out, const void* x, int64_t n, int dtype,
                                   orStream_t stream);
OPENREG_EXPORT orError_t mcpu_mul(void* out, const void* a, const void* b, int64_t n, int dtype,
                                  orStream_t stream);

/*
 * Generic kernels behind the aten registrations the reference's op-by-op
 * chains use on mcpu tensors (the router function of
 * tests/test_grouped_topk_compile.py:15-66, vLLM's native silu_and_mul and
 * rms_norm).  Strided operands of up to 8 dimensions, element strides, 0 for
 * a broadcast dimension; floating outputs compute in fp32 (fp64 for double),
 * integer outputs in int64.  Reference: csrc/aten/ops/binary_out.cpp:189-560
 * and 757-828 (add/sub/mul/div), unary_out.cpp:684-700 (masked_fill_),
 * reduction_scatter.cpp:116-150, 248-285, 461-495 (max/mean/sum),
 * topk.cpp:10-40, softmax_random_argmax.cpp:57-82, gather.cpp:10-31.
 */
enum { MCPU_BINARY_ADD = 0, MCPU_BINARY_SUB = 1, MCPU_BINARY_MUL = 2, MCPU_BINARY_DIV = 3 };
enum { MCPU_UNARY_NEG = 0, MCPU_UNARY_RSQRT = 1, MCPU_UNARY_SQRT = 2, MCPU_UNARY_POW_SCALAR = 3,
       MCPU_UNARY_BITWISE_NOT = 4, MCPU_UNARY_ABS = 5 };
enum { MCPU_REDUCE_SUM = 0, MCPU_REDUCE_MEAN = 1, MCPU_REDUCE_MAX = 2, MCPU_REDUCE_MIN = 3 };

/* out = a op (alpha * b) for add/sub, a op b otherwise. */
OPENREG_EXPORT orError_t mcpu_binary(int op, const void* a, int a_dtype, const int64_t* a_strides,
                                     const void* b, int b_dtype, const int64_t* b_strides, void* out,
                                     int out_dtype, const int64_t* out_strides, int ndim,
                                     const int64_t* sizes, double alpha, orStream_t stream);
/* out = op(x); scalar is the exponent of MCPU_UNARY_POW_SCALAR. */
OPENREG_EXPORT orError_t mcpu_unary(int op, const void* x, int x_dtype, const int64_t* x_strides,
                                    void* out, int out_dtype, const int64_t* out_strides, int ndim,
                                    const int64_t* sizes, double scalar, orStream_t stream);
/* self[i] = value where mask[i] (mask: bool, broadcast by its strides). */
OPENREG_EXPORT orError_t mcpu_masked_fill(void* self, int dtype, const int64_t* self_strides,
                                          const void* mask, const int64_t* mask_strides, int ndim,
                                          const int64_t* sizes, double fvalue, int64_t ivalue,
                                          int value_is_float, orStream_t stream);
/* Reduction of each of `rows` contiguous rows of n elements: sum, mean, or
 * max / min with the first index of the extreme (NaN propagates); indices
 * (int64, may be NULL) receive that index. */
OPENREG_EXPORT orError_t mcpu_reduce_lastdim(int op, const void* x, int dtype, int64_t rows, int64_t n,
                                             void* out, int out_dtype, int64_t* indices,
                                             orStream_t stream);
/* The k largest (largest != 0) or smallest values of each contiguous row,
 * in order, ties to the lower index, NaN counted as the largest; values
 * [rows, k] in the input dtype, indices [rows, k] int64. */
OPENREG_EXPORT orError_t mcpu_topk_lastdim(const void* x, int dtype, int64_t rows, int64_t n, int64_t k,
                                           int largest, void* values, int64_t* indices,
                                           orStream_t stream);
/* Row softmax (or log-softmax) over contiguous rows. */
OPENREG_EXPORT orError_t mcpu_softmax_lastdim(const void* x, int dtype, int64_t rows, int64_t n,
                                              void* out, int out_dtype, int log_softmax,
                                              orStream_t stream);
/* out[..] = self[.. index[..] ..] along dim; index int64; an index out of
 * range skips the element and sets the flag mcpu_device_error reports. */
OPENREG_EXPORT orError_t mcpu_gather(const void* self, int dtype, int ndim, const int64_t* self_sizes,
                                     const int64_t* self_strides, int64_t dim, const int64_t* index,
                                     const int64_t* index_sizes, const int64_t* index_strides, void* out,
                                     const int64_t* out_strides, orStream_t stream);
/* self[.. index[..] ..] = value along dim (same index rules as gather). */
OPENREG_EXPORT orError_t mcpu_scatter_value(void* self, int dtype, int ndim, const int64_t* self_sizes,
                                            const int64_t* self_strides, int64_t dim,
                                            const int64_t* index, const int64_t* index_sizes,
                                            const int64_t* index_strides, double fvalue, int64_t ivalue,
                                            int value_is_float, orStream_t stream);

#ifdef __cplusplus
}  // extern "C"
#endif
