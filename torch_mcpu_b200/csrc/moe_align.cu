// MoE expert dispatch: the per-expert token lists the fused-MoE GEMMs read,
// built from the router's topk_ids.  Same contract as vLLM's
// moe_align_block_size (vllm/_custom_ops.py:2247-2264; documented in
// vllm/model_executor/layers/fused_moe/moe_align_block_size.py:19-73):
//   sorted_token_ids  the flat indices i (token * topk + slot) of topk_ids,
//                     grouped by expert, each expert's run padded with the
//                     value numel to a multiple of block_size; here every run
//                     is in ascending i (a stable order), and every slot past
//                     the last run holds numel as well;
//   expert_ids        the expert of each block of block_size slots, -1 for
//                     the blocks past the last run;
//   num_tokens_post_pad  the number of slots the runs fill.
// The reference builds such lists, where it needs them, from scatter_add /
// index ops on host views (csrc/aten/ops/reduction_scatter.cpp:517-555).
//
// Two launches over chunks of 4096 entries (one 1024-thread CTA each):
//   count    per-chunk expert histogram (shared-memory atomics) -> counts
//   scatter  per chunk: reads every chunk's histogram (L2) for the expert
//            totals and the entries of the chunks before it, scans the
//            padded totals into run starts, builds per-warp histograms and
//            their prefix from the chunk's first slots, then each warp
//            places its 128 entries 32 at a time in index order
//            (__match_any_sync groups equal experts; rank = peers below
//            this lane), so runs come out in ascending index; then the grid
//            writes the run padding, the slots after the last run and the
//            expert of every block.
// The workspace is the [chunks, experts] int32 count matrix; every entry of
// it is written by the count launch before it is read, so it needs no
// clearing.
// Entries outside [0, num_experts) are left out and set the device error
// flag.
#include <mutex>

#include "common.cuh"

namespace mcpu {
namespace moe {

constexpr int kChunk = 4096;       // entries per chunk (one CTA)
constexpr int kThreads = 1024;     // 32 warps x 128 entries
constexpr int kWarps = kThreads / 32;
constexpr int kPerWarp = kChunk / kWarps;
constexpr int kMaxExperts = 1024;

__device__ int g_moe_error = 0;

// Workspace ints for nchunks chunks: the [nchunks, E] count matrix (at
// least one row).
inline long long workspace_ints(long long nchunks, int E) { return (nchunks > 0 ? nchunks : 1) * E; }

__global__ void __launch_bounds__(kThreads) align_count_kernel(const int32_t* __restrict__ ids, long long numel,
                                                               int E, int32_t* __restrict__ counts) {
  __shared__ int hist[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += kThreads) hist[e] = 0;
  __syncthreads();
  const long long base = static_cast<long long>(blockIdx.x) * kChunk;
  const long long left = numel - base;
  const int n = left < kChunk ? static_cast<int>(left) : kChunk;
  bool bad = false;
  int ev[kChunk / kThreads];
#pragma unroll
  for (int k = 0; k < kChunk / kThreads; ++k) {  // all loads in flight first
    const int i = threadIdx.x + k * kThreads;
    ev[k] = i < n ? __ldg(ids + base + i) : 0;
  }
#pragma unroll
  for (int k = 0; k < kChunk / kThreads; ++k) {
    if (threadIdx.x + k * kThreads >= n) continue;
    if (static_cast<unsigned>(ev[k]) < static_cast<unsigned>(E))
      atomicAdd(&hist[ev[k]], 1);
    else
      bad = true;
  }
  if (bad) atomicOr(&g_moe_error, 1);
  __syncthreads();
  int32_t* row = counts + static_cast<long long>(blockIdx.x) * E;
  for (int e = threadIdx.x; e < E; e += kThreads) row[e] = hist[e];
}

// One CTA per chunk (at least one CTA).  Every CTA reads the whole count
// matrix (all chunks' histograms, from L2) for the expert totals and for the
// entries of its own earlier chunks, scans the padded totals into run starts,
// places its chunk's entries, then the grid shares the rest of the outputs:
// the padding of each run, every slot after the last run, the expert of
// every block and (CTA 0) the slot count.
__global__ void __launch_bounds__(kThreads) align_scatter_kernel(
    const int32_t* __restrict__ ids, long long numel, int nchunks, int E, int bs,
    const int32_t* __restrict__ counts, int32_t* __restrict__ post_pad, int32_t* __restrict__ sorted,
    long long sorted_cap, int32_t* __restrict__ expert_ids, long long eid_cap) {
  extern __shared__ int smem[];  // [kWarps][E] per-warp slots | [E + 1] run starts | [P][E] x 2 partials
  int* whist = smem;
  int* start = whist + kWarps * E;
  int* ptot = start + E + 1;
  int* pbef = ptot + kThreads;
  __shared__ int scan[kThreads];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int me = blockIdx.x;
  // expert totals and the entries of chunks before this one: P threads per
  // expert, each over every P-th chunk
  const int P = kThreads / E;  // >= 1
  {
    const int e = tid % E, q = tid / E;
    int tot = 0, bef = 0;
    if (q < P) {
      int c = q;
      for (; c + 7 * P < nchunks; c += 8 * P) {  // eight loads in flight
        int v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = counts[static_cast<long long>(c + u * P) * E + e];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          tot += v[u];
          bef += c + u * P < me ? v[u] : 0;
        }
      }
      for (; c < nchunks; c += P) {
        const int v = counts[static_cast<long long>(c) * E + e];
        tot += v;
        bef += c < me ? v : 0;
      }
      ptot[q * E + e] = tot;
      pbef[q * E + e] = bef;
    }
  }
  __syncthreads();
  int total = 0, before = 0;
  if (tid < E) {
    for (int q = 0; q < P; ++q) {
      total += ptot[q * E + tid];
      before += pbef[q * E + tid];
    }
  }
  scan[tid] = tid < E ? (total + bs - 1) / bs * bs : 0;
  __syncthreads();
  for (int off = 1; off < kThreads; off <<= 1) {
    const int v = tid >= off ? scan[tid - off] : 0;
    __syncthreads();
    scan[tid] += v;
    __syncthreads();
  }
  const int end = scan[kThreads - 1];
  if (tid < E) start[tid] = tid == 0 ? 0 : scan[tid - 1];
  if (tid == 0) start[E] = end;
  if (me == 0 && tid == 0) *post_pad = end;
  // this chunk's first slot per expert, kept in the per-warp table of warp 0's
  // position until the per-warp prefix below
  int first = 0;
  if (tid < E) first = (tid == 0 ? 0 : scan[tid - 1]) + before;
  __syncthreads();
  if (me < nchunks) {
    for (int i = tid; i < kWarps * E; i += kThreads) whist[i] = 0;
    __syncthreads();
    const long long wbase = static_cast<long long>(me) * kChunk + warp * kPerWarp;
    int* wh = whist + warp * E;
    int ev[kPerWarp / 32];  // this lane's entries, loaded once (-1: none or out of range)
#pragma unroll
    for (int g = 0; g < kPerWarp / 32; ++g) {
      const long long i = wbase + g * 32 + lane;
      int e = i < numel ? __ldg(ids + i) : -1;
      if (static_cast<unsigned>(e) >= static_cast<unsigned>(E)) e = -1;
      ev[g] = e;
    }
#pragma unroll
    for (int g = 0; g < kPerWarp / 32; ++g)
      if (ev[g] >= 0) atomicAdd(&wh[ev[g]], 1);
    __syncthreads();
    if (tid < E) {
      int run = first;
      for (int w = 0; w < kWarps; ++w) {
        const int c = whist[w * E + tid];
        whist[w * E + tid] = run;
        run += c;
      }
    }
    __syncthreads();
    const unsigned below = (1u << lane) - 1u;
#pragma unroll
    for (int g = 0; g < kPerWarp / 32; ++g) {
      const long long i = wbase + g * 32 + lane;
      const int e = ev[g];
      const unsigned peers = __match_any_sync(0xFFFFFFFFu, e);
      const int rank = __popc(peers & below);
      if (e >= 0) sorted[wh[e] + rank] = static_cast<int32_t>(i);
      __syncwarp();
      if (e >= 0 && rank == 0) wh[e] += __popc(peers);
      __syncwarp();
    }
  }
  // padding of runs: expert e by CTA e % grid (its totals are in ptot/start)
  for (int e = me; e < E; e += gridDim.x) {
    int tot = 0;
    for (int q = 0; q < P; ++q) tot += ptot[q * E + e];
    const int from = start[e] + tot, to = start[e + 1];
    for (int j = from + tid; j < to; j += kThreads) sorted[j] = static_cast<int32_t>(numel);
  }
  const long long gtid = static_cast<long long>(me) * kThreads + tid;
  const long long gthreads = static_cast<long long>(gridDim.x) * kThreads;
  for (long long j = end + gtid; j < sorted_cap; j += gthreads) sorted[j] = static_cast<int32_t>(numel);
  for (long long b = gtid; b < eid_cap; b += gthreads) {
    const long long slot = b * bs;
    int ex = -1;
    if (slot < end) {
      int lo = 0, hi = E - 1;  // largest expert whose run starts at or before slot
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (start[mid] <= slot)
          lo = mid;
        else
          hi = mid - 1;
      }
      ex = lo;
    }
    expert_ids[b] = ex;
  }
}

// Checks shared by the entry points; *nchunks_out = chunks of the input.
orError_t check_args(const int32_t* topk_ids, long long numel, int E, int bs, const int32_t* sorted,
                     long long sorted_cap, const int32_t* expert_ids, long long eid_cap, const int32_t* post_pad,
                     int* nchunks_out) {
  MCPU_ARG_CHECK(numel >= 0 && numel < (1LL << 31), "moe_align_block_size: numel %lld out of range", numel);
  MCPU_ARG_CHECK(E >= 1 && E <= kMaxExperts, "moe_align_block_size: num_experts %d outside 1..%d", E,
                 kMaxExperts);
  MCPU_ARG_CHECK(bs >= 1 && bs <= (1 << 20), "moe_align_block_size: block_size %d out of range", bs);
  MCPU_ARG_CHECK(sorted && expert_ids && post_pad, "moe_align_block_size: NULL output");
  MCPU_ARG_CHECK(numel == 0 || topk_ids, "moe_align_block_size: NULL topk_ids");
  const long long a = numel + static_cast<long long>(E) * (bs - 1), b = numel * bs;
  const long long min_cap = a < b ? a : b;
  MCPU_ARG_CHECK(sorted_cap >= min_cap && sorted_cap < (1LL << 31),
                 "moe_align_block_size: sorted_token_ids holds %lld entries, %lld needed", sorted_cap, min_cap);
  MCPU_ARG_CHECK(eid_cap >= (min_cap + bs - 1) / bs,
                 "moe_align_block_size: expert_ids holds %lld entries, %lld needed", eid_cap,
                 (min_cap + bs - 1) / bs);
  *nchunks_out = static_cast<int>((numel + kChunk - 1) / kChunk);
  return orSuccess;
}

// The two launches, with `ws` as the [chunks, E] count workspace.
orError_t launch(const int32_t* topk_ids, long long numel, int E, int bs, int32_t* sorted, long long sorted_cap,
                 int32_t* expert_ids, long long eid_cap, int32_t* post_pad, int32_t* ws, int nchunks,
                 cudaStream_t st) {
  const int smem = (kWarps * E + E + 1 + 2 * kThreads) * 4;
  MCPU_CUDA_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(align_scatter_kernel),
                                   (kWarps * kMaxExperts + kMaxExperts + 1 + 2 * kThreads) * 4),
                "moe_align_block_size scatter attribute");
  if (nchunks > 0) {
    align_count_kernel<<<nchunks, kThreads, 0, st>>>(topk_ids, numel, E, ws);
    MCPU_CUDA_TRY(cudaGetLastError(), "moe_align_block_size count launch");
  }
  align_scatter_kernel<<<nchunks > 0 ? nchunks : 1, kThreads, smem, st>>>(
      topk_ids, numel, nchunks, E, bs, ws, post_pad, sorted, sorted_cap, expert_ids, eid_cap);
  MCPU_CUDA_TRY(cudaGetLastError(), "moe_align_block_size scatter launch");
  return orSuccess;
}

}  // namespace moe

orError_t moe_read_error(int* flag, bool reset) {
  MCPU_CUDA_TRY(cudaMemcpyFromSymbol(flag, moe::g_moe_error, sizeof(int)), "moe error flag");
  if (reset) {
    const int zero = 0;
    MCPU_CUDA_TRY(cudaMemcpyToSymbol(moe::g_moe_error, &zero, sizeof(int)), "moe error flag reset");
  }
  return orSuccess;
}

}  // namespace mcpu

using namespace mcpu;

extern "C" orError_t mcpu_moe_align_workspace_bytes(int64_t numel, int num_experts, uint64_t* bytes) {
  MCPU_ARG_CHECK(bytes != nullptr, "moe_align_block_size: NULL output");
  MCPU_ARG_CHECK(numel >= 0 && numel < (1LL << 31), "moe_align_block_size: numel %lld out of range",
                 static_cast<long long>(numel));
  MCPU_ARG_CHECK(num_experts >= 1 && num_experts <= moe::kMaxExperts,
                 "moe_align_block_size: num_experts %d outside 1..%d", num_experts, moe::kMaxExperts);
  const long long nchunks = (numel + moe::kChunk - 1) / moe::kChunk;
  *bytes = static_cast<uint64_t>(moe::workspace_ints(nchunks, num_experts) * 4);
  return orSuccess;
}

extern "C" orError_t mcpu_moe_align_block_size(const int32_t* topk_ids, int64_t numel, int num_experts,
                                               int block_size, int32_t* sorted_token_ids,
                                               int64_t sorted_capacity, int32_t* expert_ids,
                                               int64_t expert_ids_capacity, int32_t* num_tokens_post_pad,
                                               void* workspace, uint64_t workspace_bytes, orStream_t stream) {
  int nchunks = 0;
  orError_t e = moe::check_args(topk_ids, numel, num_experts, block_size, sorted_token_ids, sorted_capacity,
                                expert_ids, expert_ids_capacity, num_tokens_post_pad, &nchunks);
  if (e != orSuccess) return e;
  uint64_t need = 0;
  e = mcpu_moe_align_workspace_bytes(numel, num_experts, &need);
  if (e != orSuccess) return e;
  MCPU_ARG_CHECK(workspace != nullptr && workspace_bytes >= need,
                 "moe_align_block_size: workspace of %llu bytes, %llu needed",
                 static_cast<unsigned long long>(workspace_bytes), static_cast<unsigned long long>(need));
  return moe::launch(topk_ids, numel, num_experts, block_size, sorted_token_ids, sorted_capacity, expert_ids,
                     expert_ids_capacity, num_tokens_post_pad, static_cast<int32_t*>(workspace), nchunks,
                     as_cuda(stream));
}

// ---------------------------------------------------------------------------
// The same dispatch without any allocation.
//
// Some callers cannot hand this op a workspace: an inference engine that
// reserved all free device memory for its own pool when it started (a
// cudaMalloc then fails, or fragments memory the engine manages itself),
// code that must not trigger cudaMalloc's device-wide synchronisation in
// the middle of serving, and plain C callers with no device allocator of
// their own.  mcpu_moe_align_block_size_static keeps the [chunks, experts]
// count matrix in a fixed array of this library's own device memory
// instead: 65536 int32 counters (256 KiB, held on every GPU that loads the
// library until the process exits), enough for chunks x experts <= 65536
// with 4096-entry chunks, e.g. 1,048,576 entries (131072 tokens at top-8)
// with 256 experts.  Larger
// problems are rejected with an error; they need the workspace entry point.
//
// Nothing in the array has to start at zero: the count launch writes every
// counter the later launches read.  Every call shares the one array, so two
// calls whose kernels overlap on the GPU (other streams, other host
// threads) race on it; order them on one stream.
namespace {

constexpr long long kStaticCounters = 65536;
static __device__ __align__(256) int32_t g_moe_static_counts[kStaticCounters];

// Device address of the array on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up
// with cudaGetSymbolAddress once per device (on that device's first call)
// and kept.  With CUDA's lazy module loading that lookup is also what places
// the array in the device's memory, so a caller that reserves all free
// memory for its own pool makes its first call before reserving it.  The
// kept address is that of the device's current primary context; a context
// reset invalidates it.
constexpr int kMaxDevices = 64;
std::mutex g_static_mutex;
int32_t* g_static_addr[kMaxDevices] = {};

orError_t static_counts_address(int32_t** out) {
  int dev = 0;
  MCPU_CUDA_TRY(cudaGetDevice(&dev), "moe_align_block_size_static: cudaGetDevice");
  MCPU_ARG_CHECK(dev >= 0 && dev < kMaxDevices, "moe_align_block_size_static: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_static_mutex);
  if (g_static_addr[dev] == nullptr) {
    void* p = nullptr;
    MCPU_CUDA_TRY(cudaGetSymbolAddress(&p, g_moe_static_counts), "moe_align_block_size_static: cudaGetSymbolAddress");
    MCPU_ARG_CHECK(p != nullptr, "moe_align_block_size_static: no device address for the fixed scratch");
    g_static_addr[dev] = static_cast<int32_t*>(p);
  }
  *out = g_static_addr[dev];
  return orSuccess;
}

}  // namespace

extern "C" orError_t mcpu_moe_align_block_size_static(const int32_t* topk_ids, int64_t numel, int num_experts,
                                                      int block_size, int32_t* sorted_token_ids,
                                                      int64_t sorted_capacity, int32_t* expert_ids,
                                                      int64_t expert_ids_capacity, int32_t* num_tokens_post_pad,
                                                      orStream_t stream) {
  uint64_t need_bytes = 0;
  orError_t e = mcpu_moe_align_workspace_bytes(numel, num_experts, &need_bytes);  // validates numel, experts
  if (e != orSuccess) return e;
  const long long need = static_cast<long long>(need_bytes / 4);
  MCPU_ARG_CHECK(need <= kStaticCounters,
                 "moe_align_block_size_static: %lld entries over %d experts need %lld counters, the fixed "
                 "scratch holds %lld (at most %lld entries for this expert count); use mcpu_moe_align_block_size "
                 "with a workspace",
                 static_cast<long long>(numel), num_experts, need, kStaticCounters,
                 kStaticCounters / num_experts * moe::kChunk);
  int nchunks = 0;
  e = moe::check_args(topk_ids, numel, num_experts, block_size, sorted_token_ids, sorted_capacity, expert_ids,
                      expert_ids_capacity, num_tokens_post_pad, &nchunks);
  if (e != orSuccess) return e;
  int32_t* counts = nullptr;
  e = static_counts_address(&counts);
  if (e != orSuccess) return e;
  return moe::launch(topk_ids, numel, num_experts, block_size, sorted_token_ids, sorted_capacity, expert_ids,
                     expert_ids_capacity, num_tokens_post_pad, counts, nchunks, as_cuda(stream));
}
