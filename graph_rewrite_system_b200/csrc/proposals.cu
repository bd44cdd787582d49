// Source-to-xfer expansion and bounded proposal ranking (reference
// gpu_proposals.py:69-192).
//
// Semantics: each candidate (parent, source, probability) expands into the
// allowed xfers of its source in CSR order; next_gate = parent_gate + delta;
// a stable order (parent asc, next_gate asc, probability desc, xfer asc)
// keeps the first per_parent_cap actions of every parent; a stable order
// (next_gate asc, probability desc, parent_gate asc) over the survivors keeps
// the first global_cap.  Remaining ties keep expansion order.
//
// Implementation: keys are packed into 64-bit words (16-bit biased gate
// counts, order-preserving float bits, 16-bit ids) and sorted with CUB's
// stable LSD radix sort; the expansion size never leaves the device (arrays
// are sized by the host's upper bound and padded with keys that sort last).
#include <cub/cub.cuh>
#include <thrust/iterator/counting_iterator.h>

#include "grs_common.cuh"

namespace grs {

constexpr uint64_t PAD_KEY = ~0ull;
constexpr uint32_t PAD_PARENT = 0xffffffffu;

__device__ __forceinline__ uint32_t desc_float_key(float p) {
  uint32_t u = __float_as_uint(p);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // ascending order-preserving
  return ~u;                                        // descending
}

__global__ void prop_count_kernel(const int64_t* __restrict__ sources, int64_t c,
                                  const int32_t* __restrict__ xfer_counts,
                                  const int32_t* __restrict__ all_counts, int num_sources,
                                  int32_t* __restrict__ counts, int64_t* __restrict__ metrics,
                                  int32_t* __restrict__ status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int cnt = 0, all = 0;
  if (i < c) {
    const int64_t s = sources[i];
    if (s >= num_sources) {
      set_status(status, GRS_ERR_SHAPE);
    } else if (s >= 0) {  // source < 0 marks a padding row (no candidate)
      cnt = xfer_counts[s];
      all = all_counts[s];
    }
    counts[i] = cnt;
  }
  // Block-reduce the metrics (predicted, eligible) and add once per block.
  typedef cub::BlockReduce<long long, 256> Reduce;
  __shared__ typename Reduce::TempStorage t1, t2;
  const long long sa = Reduce(t1).Sum((long long)all);
  const long long sc = Reduce(t2).Sum((long long)cnt);
  if (threadIdx.x == 0) {
    atomicAdd(reinterpret_cast<unsigned long long*>(&metrics[0]), (unsigned long long)sa);
    atomicAdd(reinterpret_cast<unsigned long long*>(&metrics[1]), (unsigned long long)sc);
  }
}

__global__ void prop_expand_kernel(const int64_t* __restrict__ batch_ids,
                                   const int64_t* __restrict__ sources,
                                   const float* __restrict__ probs, int64_t c,
                                   const int32_t* __restrict__ counts,
                                   const int32_t* __restrict__ offsets,
                                   const int32_t* __restrict__ xfer_offsets,
                                   const int32_t* __restrict__ xfer_ids,
                                   const int32_t* __restrict__ gate_deltas,
                                   const int64_t* __restrict__ parent_gates, int64_t num_parents,
                                   int32_t* __restrict__ e_row, int32_t* __restrict__ e_xfer,
                                   int32_t* __restrict__ e_next, uint32_t* __restrict__ e_parent,
                                   uint64_t* __restrict__ key, int32_t* __restrict__ value,
                                   int64_t n, int32_t* __restrict__ status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= c) return;
  const int cnt = counts[i];
  if (!cnt) return;
  const int64_t parent = batch_ids[i];
  if (parent < 0 || parent >= num_parents) { set_status(status, GRS_ERR_SHAPE); return; }
  const int base = offsets[i];
  const int xo = xfer_offsets[sources[i]];
  const uint32_t pk = desc_float_key(probs[i]);
  for (int w = 0; w < cnt; ++w) {
    const int e = base + w;
    if (e >= n) { set_status(status, GRS_ERR_WORKSPACE); return; }
    const int x = xfer_ids[xo + w];
    const int64_t next = parent_gates[parent] + gate_deltas[x];
    if (next < -32768 || next > 32767 || x > 0xffff) set_status(status, GRS_ERR_SHAPE);
    e_row[e] = (int32_t)i;
    e_xfer[e] = x;
    e_next[e] = (int32_t)next;
    e_parent[e] = (uint32_t)parent;
    key[e] = ((uint64_t)(uint16_t)(next + 32768) << 48) | ((uint64_t)pk << 16) | (uint64_t)(x & 0xffff);
    value[e] = e;
  }
}

__global__ void prop_pad_kernel(const int32_t* __restrict__ total_ptr, int64_t n,
                                uint64_t* __restrict__ key, int32_t* __restrict__ value) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e < n && e >= *total_ptr) {
    key[e] = PAD_KEY;
    value[e] = (int32_t)e;
  }
}

__global__ void prop_total_kernel(const int32_t* __restrict__ counts,
                                  const int32_t* __restrict__ offsets, int64_t c,
                                  int32_t* __restrict__ total) {
  *total = c ? offsets[c - 1] + counts[c - 1] : 0;
}

__global__ void prop_parent_key_kernel(const int32_t* __restrict__ sorted_e, int64_t n,
                                       const int32_t* __restrict__ total_ptr,
                                       const uint32_t* __restrict__ e_parent,
                                       uint32_t* __restrict__ pkey) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int e = sorted_e[i];
  pkey[i] = e < *total_ptr ? e_parent[e] : PAD_PARENT;
}

// After the parent sort: rank within the parent segment; flag survivors.
__global__ void prop_segment_start_kernel(const uint32_t* __restrict__ pkey, int64_t n,
                                          int32_t* __restrict__ start) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  start[i] = (i == 0 || pkey[i] != pkey[i - 1]) ? (int32_t)i : 0;
}

__global__ void prop_flag_kernel(const uint32_t* __restrict__ pkey,
                                 const int32_t* __restrict__ seg_start, int64_t n, int cap,
                                 uint8_t* __restrict__ flags) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  flags[i] = (pkey[i] != PAD_PARENT && (int64_t)i - seg_start[i] < cap) ? 1 : 0;
}

__global__ void prop_global_key_kernel(const int32_t* __restrict__ kept_e,
                                       const int32_t* __restrict__ num_kept, int64_t m,
                                       const int32_t* __restrict__ e_next,
                                       const int32_t* __restrict__ e_row,
                                       const uint32_t* __restrict__ e_parent,
                                       const float* __restrict__ probs,
                                       const int64_t* __restrict__ parent_gates,
                                       uint64_t* __restrict__ key, int32_t* __restrict__ value,
                                       int32_t* __restrict__ status) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= m) return;
  if (j < *num_kept) {
    const int e = kept_e[j];
    const int64_t pg = parent_gates[e_parent[e]];
    if (pg < -32768 || pg > 32767) set_status(status, GRS_ERR_SHAPE);
    key[j] = ((uint64_t)(uint16_t)(e_next[e] + 32768) << 48) |
             ((uint64_t)desc_float_key(probs[e_row[e]]) << 16) |
             (uint64_t)(uint16_t)(pg + 32768);
    value[j] = e;
  } else {
    key[j] = PAD_KEY;
    value[j] = -1;
  }
}

__global__ void prop_output_kernel(const int32_t* __restrict__ sorted_e,
                                   const int32_t* __restrict__ num_kept, int64_t global_cap,
                                   const int32_t* __restrict__ e_row,
                                   const int32_t* __restrict__ e_xfer,
                                   const int32_t* __restrict__ e_next,
                                   int64_t* __restrict__ out_row, int64_t* __restrict__ out_xfer,
                                   int64_t* __restrict__ out_next, int64_t* __restrict__ out_count) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t count = min((int64_t)*num_kept, global_cap);
  if (j == 0) *out_count = count;
  if (j >= global_cap) return;
  if (j < count) {
    const int e = sorted_e[j];
    out_row[j] = e_row[e];
    out_xfer[j] = e_xfer[e];
    out_next[j] = e_next[e];
  } else {
    out_row[j] = -1;
    out_xfer[j] = -1;
    out_next[j] = 0;
  }
}

struct PropWorkspace {
  // element arrays
  int32_t *counts, *offsets, *total, *num_kept;
  int32_t *e_row, *e_xfer, *e_next, *seg_start;
  uint32_t *e_parent, *pkey_in, *pkey_out;
  uint64_t *key_in, *key_out;
  int32_t *val_in, *val_out, *kept;
  uint8_t* flags;
  void* cub_tmp;
  size_t cub_bytes;
};

static size_t align_up(size_t v) { return (v + 255) & ~size_t(255); }

// Lay out (or measure, when base == nullptr) the workspace.
static size_t prop_layout(char* base, int64_t c, int64_t n, PropWorkspace* w) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> char* {
    char* p = base ? base + off : nullptr;
    off += align_up(bytes);
    return p;
  };
  const int64_t cc = c > 0 ? c : 1, nn = n > 0 ? n : 1;
  w->counts = (int32_t*)take(cc * 4);
  w->offsets = (int32_t*)take(cc * 4);
  w->total = (int32_t*)take(4);
  w->num_kept = (int32_t*)take(4);
  w->e_row = (int32_t*)take(nn * 4);
  w->e_xfer = (int32_t*)take(nn * 4);
  w->e_next = (int32_t*)take(nn * 4);
  w->seg_start = (int32_t*)take(nn * 4);
  w->e_parent = (uint32_t*)take(nn * 4);
  w->pkey_in = (uint32_t*)take(nn * 4);
  w->pkey_out = (uint32_t*)take(nn * 4);
  w->key_in = (uint64_t*)take(nn * 8);
  w->key_out = (uint64_t*)take(nn * 8);
  w->val_in = (int32_t*)take(nn * 4);
  w->val_out = (int32_t*)take(nn * 4);
  w->kept = (int32_t*)take(nn * 4);
  w->flags = (uint8_t*)take(nn);
  // CUB temporary storage: the largest requirement of the calls below.
  size_t need = 0, t = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, t, (int32_t*)nullptr, (int32_t*)nullptr, (int)cc);
  need = t > need ? t : need;
  cub::DeviceRadixSort::SortPairs(nullptr, t, (uint64_t*)nullptr, (uint64_t*)nullptr,
                                  (int32_t*)nullptr, (int32_t*)nullptr, (int)nn);
  need = t > need ? t : need;
  cub::DeviceRadixSort::SortPairs(nullptr, t, (uint32_t*)nullptr, (uint32_t*)nullptr,
                                  (int32_t*)nullptr, (int32_t*)nullptr, (int)nn);
  need = t > need ? t : need;
  cub::DeviceScan::InclusiveScan(nullptr, t, (int32_t*)nullptr, (int32_t*)nullptr,
                                 cub::Max(), (int)nn);
  need = t > need ? t : need;
  cub::DeviceSelect::Flagged(nullptr, t, (int32_t*)nullptr, (uint8_t*)nullptr,
                             (int32_t*)nullptr, (int32_t*)nullptr, (int)nn);
  need = t > need ? t : need;
  w->cub_bytes = need;
  w->cub_tmp = take(need);
  return off;
}

}  // namespace grs

using namespace grs;

extern "C" int64_t grs_proposals_workspace_bytes(int64_t max_candidates, int64_t max_expanded) {
  PropWorkspace w;
  return (int64_t)prop_layout(nullptr, max_candidates, max_expanded, &w);
}

extern "C" int grs_proposals_rank(
    const int64_t* batch_ids, const int64_t* sources, const float* probabilities,
    int64_t num_candidates, const int64_t* parent_gate_counts, int64_t num_parents,
    const int32_t* xfer_offsets, const int32_t* xfer_counts, const int32_t* xfer_ids,
    const int32_t* gate_deltas, const int32_t* all_xfer_counts, int num_sources,
    int64_t max_expanded, int per_parent_cap, int64_t global_cap, int64_t* out_row,
    int64_t* out_xfer, int64_t* out_next_gate, int64_t* out_count, int64_t* out_metrics,
    void* workspace, int64_t workspace_bytes, int32_t* status, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (num_candidates < 0 || max_expanded < 0 || per_parent_cap < 0 || global_cap < 0 ||
      num_candidates > (1ll << 30) || max_expanded > (1ll << 30))
    return GRS_ERR_SHAPE;
  PropWorkspace w;
  const int64_t need = (int64_t)prop_layout((char*)workspace, num_candidates, max_expanded, &w);
  if (need > workspace_bytes) return GRS_ERR_WORKSPACE;
  const int64_t c = num_candidates, n = max_expanded;
  cudaMemsetAsync(out_metrics, 0, 2 * sizeof(int64_t), s);
  if (c == 0 || n == 0) {
    cudaMemsetAsync(out_count, 0, sizeof(int64_t), s);
    GRS_CUDA_CHECK_LAUNCH();
    return GRS_OK;
  }
  const int T = 256;
  prop_count_kernel<<<ceil_div(c, T), T, 0, grs::counted(s)>>>(sources, c, xfer_counts, all_xfer_counts,
                                                 num_sources, w.counts, out_metrics, status);
  size_t tb = w.cub_bytes;
  cub::DeviceScan::ExclusiveSum(w.cub_tmp, tb, w.counts, w.offsets, (int)c, s);
  prop_total_kernel<<<1, 1, 0, grs::counted(s)>>>(w.counts, w.offsets, c, w.total);
  prop_expand_kernel<<<ceil_div(c, T), T, 0, grs::counted(s)>>>(
      batch_ids, sources, probabilities, c, w.counts, w.offsets, xfer_offsets, xfer_ids,
      gate_deltas, parent_gate_counts, num_parents, w.e_row, w.e_xfer, w.e_next, w.e_parent,
      w.key_in, w.val_in, n, status);
  prop_pad_kernel<<<ceil_div(n, T), T, 0, grs::counted(s)>>>(w.total, n, w.key_in, w.val_in);
  // (next_gate, prob desc, xfer) then stable by parent.
  tb = w.cub_bytes;
  cub::DeviceRadixSort::SortPairs(w.cub_tmp, tb, w.key_in, w.key_out, w.val_in, w.val_out,
                                  (int)n, 0, 64, s);
  prop_parent_key_kernel<<<ceil_div(n, T), T, 0, grs::counted(s)>>>(w.val_out, n, w.total, w.e_parent,
                                                      w.pkey_in);
  tb = w.cub_bytes;
  cub::DeviceRadixSort::SortPairs(w.cub_tmp, tb, w.pkey_in, w.pkey_out, w.val_out, w.val_in,
                                  (int)n, 0, 32, s);
  prop_segment_start_kernel<<<ceil_div(n, T), T, 0, grs::counted(s)>>>(w.pkey_out, n, w.seg_start);
  tb = w.cub_bytes;
  cub::DeviceScan::InclusiveScan(w.cub_tmp, tb, w.seg_start, w.val_out, cub::Max(), (int)n, s);
  prop_flag_kernel<<<ceil_div(n, T), T, 0, grs::counted(s)>>>(w.pkey_out, w.val_out, n, per_parent_cap,
                                                w.flags);
  tb = w.cub_bytes;
  cub::DeviceSelect::Flagged(w.cub_tmp, tb, w.val_in, w.flags, w.kept, w.num_kept, (int)n, s);
  prop_global_key_kernel<<<ceil_div(n, T), T, 0, grs::counted(s)>>>(w.kept, w.num_kept, n, w.e_next, w.e_row,
                                                      w.e_parent, probabilities,
                                                      parent_gate_counts, w.key_in, w.val_in,
                                                      status);
  tb = w.cub_bytes;
  cub::DeviceRadixSort::SortPairs(w.cub_tmp, tb, w.key_in, w.key_out, w.val_in, w.val_out,
                                  (int)n, 0, 64, s);
  if (global_cap > 0)
    prop_output_kernel<<<ceil_div(global_cap, T), T, 0, grs::counted(s)>>>(
        w.val_out, w.num_kept, global_cap, w.e_row, w.e_xfer, w.e_next, out_row, out_xfer,
        out_next_gate, out_count);
  else
    cudaMemsetAsync(out_count, 0, sizeof(int64_t), s);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free proposal ranking.
//
// grs_proposals_rank needs a scratch workspace that its caller allocates.
// Some callers cannot allocate device memory at the moment they rank
// proposals: a host runtime whose device memory is entirely reserved up front
// by its own pool, a foreign-language binding (Go, Java, Rust) that has no
// handle on the framework's caching allocator, or a latency-critical loop in
// which a cudaMalloc would synchronise the device.  For them this variant
// takes its scratch from a fixed array compiled into the library:
// GRS_PROPOSALS_STATIC_SCRATCH_BYTES (8 MiB) of device memory that every GPU
// which loads this code keeps until the process exits.
//
// The array is named here as a host-side stand-in; its device address is
// resolved with cudaGetSymbolAddress once per device, on that device's first
// call (so make the first call on each device before any stream capture).
// All calls share the one array, which keeps whatever the last call left in
// it; every scratch location is written before it is read, so no clearing is
// needed, but two calls whose work overlaps on the GPU (different streams
// without ordering between them) race on the array.
// ---------------------------------------------------------------------------
#include <mutex>

namespace grs {
constexpr int64_t kProposalStaticScratchBytes = GRS_PROPOSALS_STATIC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_proposal_scratch[kProposalStaticScratchBytes];
constexpr int kMaxDevices = 64;
}  // namespace grs

extern "C" int grs_proposals_rank_static(
    const int64_t* batch_ids, const int64_t* sources, const float* probabilities,
    int64_t num_candidates, const int64_t* parent_gate_counts, int64_t num_parents,
    const int32_t* xfer_offsets, const int32_t* xfer_counts, const int32_t* xfer_ids,
    const int32_t* gate_deltas, const int32_t* all_xfer_counts, int num_sources,
    int64_t max_expanded, int per_parent_cap, int64_t global_cap, int64_t* out_row,
    int64_t* out_xfer, int64_t* out_next_gate, int64_t* out_count, int64_t* out_metrics,
    int32_t* status, void* stream) {
  if (num_candidates < 0 || max_expanded < 0 || num_candidates > (1ll << 30) ||
      max_expanded > (1ll << 30))
    return GRS_ERR_SHAPE;
  PropWorkspace w;
  if ((int64_t)prop_layout(nullptr, num_candidates, max_expanded, &w) >
      kProposalStaticScratchBytes)
    return GRS_ERR_TOO_LARGE;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices)
    return GRS_ERR_CUDA;
  static std::mutex lock;
  static void* scratch_address[kMaxDevices] = {};
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> guard(lock);
    if (scratch_address[device] == nullptr) {
      void* address = nullptr;
      if (cudaGetSymbolAddress(&address, g_proposal_scratch) != cudaSuccess || !address)
        return GRS_ERR_CUDA;
      scratch_address[device] = address;
    }
    scratch = scratch_address[device];
  }
  return grs_proposals_rank(batch_ids, sources, probabilities, num_candidates,
                            parent_gate_counts, num_parents, xfer_offsets, xfer_counts,
                            xfer_ids, gate_deltas, all_xfer_counts, num_sources, max_expanded,
                            per_parent_cap, global_cap, out_row, out_xfer, out_next_gate,
                            out_count, out_metrics, scratch, kProposalStaticScratchBytes, status,
                            stream);
}

// ---------------------------------------------------------------------------
// Parent-grouped ranking.  When the candidates of parent b are the rows
// [b*k, (b+1)*k) (the padded layout of the device candidate selection, rows
// with source < 0 are absent), the per-parent cap needs no global sort: one
// CTA per parent expands its candidates in row order, sorts the expansion in
// shared memory by (next gate, probability desc, xfer, expansion index) - the
// key order of gpu_proposals.py:128-135 with the stable sort's tie rule - and
// keeps the first per_parent_cap.  The concatenation of the per-parent lists
// in parent order is exactly the order the reference's stable global sort
// sees, so one stable radix sort of <= parents*cap packed keys finishes.
// ---------------------------------------------------------------------------
namespace grs {

constexpr int GRP_THREADS = 512;
constexpr int GRP_MAX_EXPANDED = 4096;

__global__ void __launch_bounds__(GRP_THREADS) prop_grouped_parent_kernel(
    const int64_t* __restrict__ sources, const float* __restrict__ probs, int k,
    const int64_t* __restrict__ parent_gates, const int32_t* __restrict__ xfer_offsets,
    const int32_t* __restrict__ xfer_counts, const int32_t* __restrict__ xfer_ids,
    const int32_t* __restrict__ gate_deltas, const int32_t* __restrict__ all_counts,
    int num_sources, int cap, int32_t* __restrict__ sel_row, int32_t* __restrict__ sel_xfer,
    int32_t* __restrict__ sel_next, int64_t* __restrict__ metrics, int32_t* __restrict__ status) {
  extern __shared__ unsigned long long keys[];   // [GRP_MAX_EXPANDED]
  __shared__ int warp_tot[GRP_THREADS / 32];
  __shared__ int s_base;
  __shared__ unsigned long long s_pred, s_elig;
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) { s_base = 0; s_pred = 0; s_elig = 0; }
  __syncthreads();
  const int64_t pgate = parent_gates[b];
  // expansion in row order: block scan of the per-row xfer counts
  for (int r0 = 0; r0 < k; r0 += GRP_THREADS) {
    const int r = r0 + tid;
    int cnt = 0, all = 0;
    int64_t src = -1;
    if (r < k) {
      src = sources[(int64_t)b * k + r];
      if (src >= num_sources) { set_status(status, GRS_ERR_SHAPE); src = -1; }
      if (src >= 0) { cnt = xfer_counts[src]; all = all_counts[src]; }
    }
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int before = s_base;
    for (int w = 0; w < warp; ++w) before += warp_tot[w];
    const int start = before + incl - cnt;
    if (cnt) {
      atomicAdd(&s_pred, (unsigned long long)all);
      atomicAdd(&s_elig, (unsigned long long)cnt);
      const uint32_t pk = desc_float_key(probs[(int64_t)b * k + r]);
      const int xo = xfer_offsets[src];
      for (int w = 0; w < cnt; ++w) {
        const int e = start + w;
        if (e >= GRP_MAX_EXPANDED) { set_status(status, GRS_ERR_WORKSPACE); break; }
        const int x = xfer_ids[xo + w];
        const int delta = gate_deltas[x];
        if (delta < -8 || delta > 7 || x > 0xffff) set_status(status, GRS_ERR_SHAPE);
        keys[e] = ((unsigned long long)(uint32_t)(delta + 8) << 60) |
                  ((unsigned long long)pk << 28) | ((unsigned long long)(x & 0xffff) << 12) |
                  (unsigned long long)(e & 0xfff);
      }
    } else if (all) {
      atomicAdd(&s_pred, (unsigned long long)all);
    }
    __syncthreads();
    if (tid == 0) {
      int tot = 0;
      for (int w = 0; w < GRP_THREADS / 32; ++w) tot += warp_tot[w];
      s_base += tot;
    }
    __syncthreads();
  }
  const int n = min(s_base, GRP_MAX_EXPANDED);
  // Expansion index -> candidate row, from a second walk over the rows.
  __shared__ int16_t row_of[GRP_MAX_EXPANDED];
  __syncthreads();  // every thread has read s_base before it is reset
  if (tid == 0) s_base = 0;
  __syncthreads();
  for (int r0 = 0; r0 < k; r0 += GRP_THREADS) {
    const int r = r0 + tid;
    int cnt = 0;
    if (r < k) {
      const int64_t src = sources[(int64_t)b * k + r];
      if (src >= 0 && src < num_sources) cnt = xfer_counts[src];
    }
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int before = s_base;
    for (int w = 0; w < warp; ++w) before += warp_tot[w];
    for (int w = 0; w < cnt; ++w) {
      const int e = before + incl - cnt + w;
      if (e < GRP_MAX_EXPANDED) row_of[e] = (int16_t)r;
    }
    __syncthreads();
    if (tid == 0) {
      int tot = 0;
      for (int w = 0; w < GRP_THREADS / 32; ++w) tot += warp_tot[w];
      s_base += tot;
    }
    __syncthreads();
  }
  int size = 1;
  while (size < n) size <<= 1;
  for (int i = n + tid; i < size; i += GRP_THREADS) keys[i] = ~0ull;
  __syncthreads();
  for (int k2 = 2; k2 <= size; k2 <<= 1) {
    for (int j = k2 >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < size; i += GRP_THREADS) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long x = keys[i], y = keys[l];
          const bool asc = (i & k2) == 0;
          if (asc ? (x > y) : (x < y)) { keys[i] = y; keys[l] = x; }
        }
      }
      __syncthreads();
    }
  }
  const int keep = min(n, cap);
  for (int r = tid; r < cap; r += GRP_THREADS) {
    const int64_t o = (int64_t)b * cap + r;
    if (r < keep) {
      const unsigned long long key = keys[r];
      const int e = (int)(key & 0xfff);
      const int x = (int)((key >> 12) & 0xffff);
      const int delta = (int)(key >> 60) - 8;
      sel_row[o] = b * k + row_of[e];
      sel_xfer[o] = x;
      sel_next[o] = (int32_t)(pgate + delta);
    } else {
      sel_row[o] = -1;
      sel_xfer[o] = -1;
      sel_next[o] = 0;
    }
  }
  if (tid == 0) {
    atomicAdd(reinterpret_cast<unsigned long long*>(&metrics[0]), s_pred);
    atomicAdd(reinterpret_cast<unsigned long long*>(&metrics[1]), s_elig);
  }
}

__global__ void prop_grouped_key_kernel(const int32_t* __restrict__ sel_row,
                                        const int32_t* __restrict__ sel_next,
                                        const float* __restrict__ probs,
                                        const int64_t* __restrict__ parent_gates, int k,
                                        int64_t n, uint64_t* __restrict__ key,
                                        int32_t* __restrict__ value, int32_t* __restrict__ status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t row = sel_row[i];
  if (row < 0) {
    key[i] = PAD_KEY;
  } else {
    const int64_t pg = parent_gates[row / k];
    const int32_t next = sel_next[i];
    if (pg < -32768 || pg > 32767 || next < -32768 || next > 32767) set_status(status, GRS_ERR_SHAPE);
    key[i] = ((uint64_t)(uint16_t)(next + 32768) << 48) |
             ((uint64_t)desc_float_key(probs[row]) << 16) | (uint64_t)(uint16_t)(pg + 32768);
  }
  value[i] = (int32_t)i;
}

__global__ void prop_grouped_output_kernel(const uint64_t* __restrict__ sorted_key,
                                           const int32_t* __restrict__ sorted_pos,
                                           int64_t global_cap, const int32_t* __restrict__ sel_row,
                                           const int32_t* __restrict__ sel_xfer,
                                           const int32_t* __restrict__ sel_next, int64_t n,
                                           int64_t* __restrict__ out_row,
                                           int64_t* __restrict__ out_xfer,
                                           int64_t* __restrict__ out_next,
                                           int64_t* __restrict__ out_count) {
  __shared__ int block_count;
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (threadIdx.x == 0) block_count = 0;
  __syncthreads();
  bool live = j < global_cap && j < n && sorted_key[j] != PAD_KEY;
  if (j < global_cap) {
    if (live) {
      const int32_t pos = sorted_pos[j];
      out_row[j] = sel_row[pos];
      out_xfer[j] = sel_xfer[pos];
      out_next[j] = sel_next[pos];
    } else {
      out_row[j] = -1;
      out_xfer[j] = -1;
      out_next[j] = 0;
    }
  }
  if (live) atomicAdd(&block_count, 1);
  __syncthreads();
  if (threadIdx.x == 0 && block_count)
    atomicAdd(reinterpret_cast<unsigned long long*>(out_count), (unsigned long long)block_count);
}

}  // namespace grs

extern "C" int64_t grs_proposals_grouped_workspace_bytes(int64_t parents, int per_parent_cap) {
  const int64_t n = parents * (int64_t)per_parent_cap;
  size_t t = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, t, (uint64_t*)nullptr, (uint64_t*)nullptr,
                                  (int32_t*)nullptr, (int32_t*)nullptr, (int)(n > 0 ? n : 1));
  const size_t elems = (size_t)(n > 0 ? n : 1);
  return (int64_t)(align_up(elems * 4) * 3 + align_up(elems * 8) * 2 + align_up(elems * 4) * 2 +
                   align_up(t));
}

extern "C" int grs_proposals_rank_grouped(
    const int64_t* sources, const float* probabilities, int64_t parents, int k,
    const int64_t* parent_gate_counts, const int32_t* xfer_offsets, const int32_t* xfer_counts,
    const int32_t* xfer_ids, const int32_t* gate_deltas, const int32_t* all_xfer_counts,
    int num_sources, int per_parent_cap, int64_t global_cap, int64_t* out_row, int64_t* out_xfer,
    int64_t* out_next_gate, int64_t* out_count, int64_t* out_metrics, void* workspace,
    int64_t workspace_bytes, int32_t* status, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (parents < 0 || k <= 0 || per_parent_cap <= 0 || global_cap < 0 ||
      per_parent_cap > GRP_MAX_EXPANDED)
    return GRS_ERR_SHAPE;
  if (grs_proposals_grouped_workspace_bytes(parents, per_parent_cap) > workspace_bytes)
    return GRS_ERR_WORKSPACE;
  cudaMemsetAsync(out_metrics, 0, 2 * sizeof(int64_t), s);
  cudaMemsetAsync(out_count, 0, sizeof(int64_t), s);
  if (parents == 0) {
    GRS_CUDA_CHECK_LAUNCH();
    return GRS_OK;
  }
  const int64_t n = parents * per_parent_cap;
  char* base = (char*)workspace;
  size_t off = 0;
  auto take = [&](size_t bytes) { char* p = base + off; off += align_up(bytes); return p; };
  int32_t* sel_row = (int32_t*)take(n * 4);
  int32_t* sel_xfer = (int32_t*)take(n * 4);
  int32_t* sel_next = (int32_t*)take(n * 4);
  uint64_t* key_in = (uint64_t*)take(n * 8);
  uint64_t* key_out = (uint64_t*)take(n * 8);
  int32_t* val_in = (int32_t*)take(n * 4);
  int32_t* val_out = (int32_t*)take(n * 4);
  size_t tb = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, tb, key_in, key_out, val_in, val_out, (int)n);
  void* cub_tmp = take(tb);
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(prop_grouped_parent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         GRP_MAX_EXPANDED * 8);
    attr[dev] = true;
  }
  prop_grouped_parent_kernel<<<(unsigned)parents, GRP_THREADS, GRP_MAX_EXPANDED * 8, grs::counted(s)>>>(
      sources, probabilities, k, parent_gate_counts, xfer_offsets, xfer_counts, xfer_ids,
      gate_deltas, all_xfer_counts, num_sources, per_parent_cap, sel_row, sel_xfer, sel_next,
      out_metrics, status);
  prop_grouped_key_kernel<<<ceil_div(n, 256), 256, 0, grs::counted(s)>>>(sel_row, sel_next, probabilities,
                                                           parent_gate_counts, k, n, key_in,
                                                           val_in, status);
  cub::DeviceRadixSort::SortPairs(cub_tmp, tb, key_in, key_out, val_in, val_out, (int)n, 0, 64,
                                  s);
  if (global_cap > 0)
    prop_grouped_output_kernel<<<ceil_div(global_cap, 256), 256, 0, grs::counted(s)>>>(
        key_out, val_out, global_cap, sel_row, sel_xfer, sel_next, n, out_row, out_xfer,
        out_next_gate, out_count);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

// ---------------------------------------------------------------------------
// Proposals from a primary and an exploration model with a per-parent quota
// (build_legacy_proposals, paged_rollout_benchmark.py:101-210; the search uses
// it while a second model is loaded, :917-919, 937-961).
//
// The candidate table is the primary model's rows [0, c_primary) followed by
// the exploration model's rows.  Per parent, each model's actions are ranked
// (next gate, probability desc, xfer, expansion order); the parent keeps the
// first cap - quota primary actions, then exploration actions whose
// (xfer, anchor, binding) is not already kept - appending before checking
// the cap, as the reference does - then the remaining primary actions that
// are not duplicates, up to the cap.  An xfer fixes its source and both
// models decode bindings on the same topology, so two actions share
// (xfer, anchor, binding) exactly when their candidates share (parent,
// source, anchor): a hash join of the two tables on that key pairs them.
// The survivors are ordered by (next gate, probability desc, parent gate)
// with ties in the order the parent's list is sorted by (next gate,
// probability desc, xfer, position in the kept list) - two stable radix
// sorts.
// ---------------------------------------------------------------------------
namespace grs {

__global__ void prop_count_models_kernel(const int64_t* __restrict__ sources, int64_t c,
                                         int64_t c_primary, const int32_t* __restrict__ xfer_counts,
                                         const int32_t* __restrict__ all_counts, int num_sources,
                                         int32_t* __restrict__ counts, int64_t* __restrict__ metrics,
                                         int32_t* __restrict__ status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  long long v[4] = {0, 0, 0, 0};   // primary predicted, eligible; exploration predicted, eligible
  if (i < c) {
    const int64_t s = sources[i];
    int cnt = 0, all = 0;
    if (s >= num_sources) {
      set_status(status, GRS_ERR_SHAPE);
    } else if (s >= 0) {
      cnt = xfer_counts[s];
      all = all_counts[s];
    }
    counts[i] = cnt;
    const int m = i >= c_primary ? 2 : 0;
    v[m] = all;
    v[m + 1] = cnt;
  }
  typedef cub::BlockReduce<long long, 256> Reduce;
  __shared__ typename Reduce::TempStorage t[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const long long sum = Reduce(t[k]).Sum(v[k]);
    if (threadIdx.x == 0 && sum)
      atomicAdd(reinterpret_cast<unsigned long long*>(&metrics[k]), (unsigned long long)sum);
  }
}

__global__ void prop_model_key_kernel(const int32_t* __restrict__ sorted_e, int64_t n,
                                      const int32_t* __restrict__ total_ptr,
                                      const uint32_t* __restrict__ e_parent,
                                      const int32_t* __restrict__ e_row, int64_t c_primary,
                                      uint32_t* __restrict__ pkey) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int e = sorted_e[i];
  pkey[i] = e < *total_ptr ? e_parent[e] * 2u + (e_row[e] >= c_primary ? 1u : 0u) : PAD_PARENT;
}

// after the (parent, model) sort: every action's position and the bounds
// of every (parent, model) segment (bounds preset to 0: empty)
__global__ void prop_positions_kernel(const uint32_t* __restrict__ pkey,
                                      const int32_t* __restrict__ sorted_e, int64_t n,
                                      int32_t* __restrict__ pos_of, int32_t* __restrict__ seg_begin,
                                      int32_t* __restrict__ seg_end) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t k = pkey[i];
  if (k == PAD_PARENT) return;
  pos_of[sorted_e[i]] = (int32_t)i;
  if (i == 0 || pkey[i - 1] != k) seg_begin[k] = (int32_t)i;
  if (i == n - 1 || pkey[i + 1] != k) seg_end[k] = (int32_t)(i + 1);
}

__device__ __forceinline__ bool candidate_key(int64_t parent, int64_t source, int64_t anchor,
                                              uint64_t* key) {
  if (parent < 0 || parent >= (1ll << 23) || source < 0 || source >= (1ll << 12) || anchor < 0 ||
      anchor >= (1ll << 28))
    return false;
  *key = (((uint64_t)parent << 40) | ((uint64_t)source << 28) | (uint64_t)anchor) + 1;
  return true;
}

// primary rows into an open-addressing table keyed by (parent, source, anchor)
__global__ void prop_join_insert_kernel(const int64_t* __restrict__ batch_ids,
                                        const int64_t* __restrict__ sources,
                                        const int64_t* __restrict__ anchors, int64_t c_primary,
                                        unsigned long long* __restrict__ hkeys,
                                        int32_t* __restrict__ hvals, int64_t hmask,
                                        int32_t* __restrict__ match_e, int32_t* __restrict__ status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= c_primary) return;
  match_e[i] = -1;
  if (sources[i] < 0) return;
  uint64_t key;
  if (!candidate_key(batch_ids[i], sources[i], anchors[i], &key)) {
    set_status(status, GRS_ERR_SHAPE);
    return;
  }
  int64_t slot = (int64_t)(mix64(key) & (uint64_t)hmask);
  for (int64_t probe = 0; probe <= hmask; ++probe, slot = (slot + 1) & hmask) {
    const unsigned long long prev = atomicCAS(&hkeys[slot], 0ull, (unsigned long long)key);
    if (prev == 0ull) {
      hvals[slot] = (int32_t)i;
      return;
    }
    if (prev == (unsigned long long)key) return;   // the first row of a repeated key wins
  }
  set_status(status, GRS_ERR_WORKSPACE);
}

// exploration rows look up their primary partner (and tell it theirs)
__global__ void prop_join_lookup_kernel(const int64_t* __restrict__ batch_ids,
                                        const int64_t* __restrict__ sources,
                                        const int64_t* __restrict__ anchors, int64_t c_primary,
                                        int64_t c, const unsigned long long* __restrict__ hkeys,
                                        const int32_t* __restrict__ hvals, int64_t hmask,
                                        int32_t* __restrict__ match_p, int32_t* __restrict__ match_e) {
  const int64_t i = c_primary + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= c) return;
  match_p[i - c_primary] = -1;
  uint64_t key;
  if (sources[i] < 0 || !candidate_key(batch_ids[i], sources[i], anchors[i], &key)) return;
  int64_t slot = (int64_t)(mix64(key) & (uint64_t)hmask);
  for (int64_t probe = 0; probe <= hmask; ++probe, slot = (slot + 1) & hmask) {
    const unsigned long long k = hkeys[slot];
    if (k == 0ull) return;
    if (k == (unsigned long long)key) {
      const int32_t row = hvals[slot];
      match_p[i - c_primary] = row;
      match_e[row] = (int32_t)i;
      return;
    }
  }
}

constexpr int EXPL_THREADS = 256;

// one CTA per parent: the kept list (positions in spos) of the quota rule
__global__ void __launch_bounds__(EXPL_THREADS) prop_select_exploration_kernel(
    const int32_t* __restrict__ sorted_e, const int32_t* __restrict__ pos_of,
    const int32_t* __restrict__ seg_begin, const int32_t* __restrict__ seg_end,
    const int32_t* __restrict__ e_row, const int32_t* __restrict__ offsets, int64_t c_primary,
    const int32_t* __restrict__ match_p, const int32_t* __restrict__ match_e, int cap, int quota,
    uint8_t* __restrict__ keep, uint8_t* __restrict__ taken_e, int32_t* __restrict__ spos,
    int64_t* __restrict__ metrics) {
  typedef cub::BlockScan<int, EXPL_THREADS> Scan;
  __shared__ typename Scan::TempStorage scan;
  const int64_t p = blockIdx.x;
  const int tid = threadIdx.x;
  const int ps = seg_begin[2 * p], pe = seg_end[2 * p];
  const int es = seg_begin[2 * p + 1], ee = seg_end[2 * p + 1];
  const int np = pe - ps, ne = ee - es;
  const int limit = cap - min(quota, cap);          // primary actions kept first
  const int n0 = min(limit, np);
  for (int i = tid; i < n0; i += EXPL_THREADS) {
    const int e = sorted_e[ps + i];
    keep[e] = 1;
    spos[e] = i;
  }
  // exploration actions: the reference appends, then checks the cap, so a
  // full primary head still admits one
  const int want = n0 >= cap ? 1 : cap - n0;
  int taken = 0;
  for (int base = 0; base < ne && taken < want; base += EXPL_THREADS) {
    const int i = base + tid;
    int ok = 0, e = -1;
    if (i < ne) {
      e = sorted_e[es + i];
      const int row = e_row[e];
      const int rp = match_p[row - c_primary];
      bool dup = false;
      if (rp >= 0) dup = pos_of[offsets[rp] + (e - offsets[row])] - ps < limit;
      ok = dup ? 0 : 1;
    }
    int prefix, total;
    Scan(scan).ExclusiveSum(ok, prefix, total);
    if (ok && taken + prefix < want) {
      keep[e] = 1;
      taken_e[e] = 1;
      spos[e] = n0 + taken + prefix;
    }
    taken += min(total, want - taken);
    __syncthreads();
  }
  // the remaining primary actions that no kept exploration action repeats
  const int kept = n0 + taken;
  if (kept < cap) {
    const int need = cap - kept;
    int filled = 0;
    for (int base = limit; base < np && filled < need; base += EXPL_THREADS) {
      const int i = base + tid;
      int ok = 0, e = -1;
      if (i < np) {
        e = sorted_e[ps + i];
        const int row = e_row[e];
        const int re = match_e[row];
        bool dup = false;
        if (re >= 0) dup = taken_e[offsets[re] + (e - offsets[row])] != 0;
        ok = dup ? 0 : 1;
      }
      int prefix, total;
      Scan(scan).ExclusiveSum(ok, prefix, total);
      if (ok && filled + prefix < need) {
        keep[e] = 1;
        spos[e] = kept + filled + prefix;
      }
      filled += min(total, need - filled);
      __syncthreads();
    }
  }
  if (tid == 0 && taken)
    atomicAdd(reinterpret_cast<unsigned long long*>(&metrics[4]), (unsigned long long)taken);
}

// keys of the final order: secondary (parent, xfer, kept position), primary
// (next gate, probability desc, parent gate)
__global__ void prop_exploration_keys_kernel(
    const int32_t* __restrict__ kept_e, const int32_t* __restrict__ num_kept, int64_t m,
    const int32_t* __restrict__ e_next, const int32_t* __restrict__ e_row,
    const int32_t* __restrict__ e_xfer, const uint32_t* __restrict__ e_parent,
    const int32_t* __restrict__ spos, const float* __restrict__ probs,
    const int64_t* __restrict__ parent_gates, uint64_t* __restrict__ key2,
    uint64_t* __restrict__ key1, int32_t* __restrict__ value, int32_t* __restrict__ status) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= m) return;
  if (j < *num_kept) {
    const int e = kept_e[j];
    const uint32_t parent = e_parent[e];
    const int64_t pg = parent_gates[parent];
    if (pg < -32768 || pg > 32767 || parent >= (1u << 24) || spos[e] > 0xffff)
      set_status(status, GRS_ERR_SHAPE);
    key2[j] = ((uint64_t)parent << 32) | ((uint64_t)(e_xfer[e] & 0xffff) << 16) |
              (uint64_t)(spos[e] & 0xffff);
    key1[j] = ((uint64_t)(uint16_t)(e_next[e] + 32768) << 48) |
              ((uint64_t)desc_float_key(probs[e_row[e]]) << 16) | (uint64_t)(uint16_t)(pg + 32768);
    value[j] = (int32_t)j;
  } else {
    key2[j] = PAD_KEY;
    key1[j] = PAD_KEY;
    value[j] = -1;
  }
}

// after the tie-order sort (order[i] = kept index): the ranking keys and
// the action ids in that order
__global__ void prop_gather_keys_kernel(const int32_t* __restrict__ order, int64_t n,
                                        const int32_t* __restrict__ kept_e,
                                        const int32_t* __restrict__ num_kept,
                                        const uint64_t* __restrict__ key1,
                                        uint64_t* __restrict__ key_out,
                                        int32_t* __restrict__ e_out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int j = order[i];
  if (j >= 0 && j < *num_kept) {
    key_out[i] = key1[j];
    e_out[i] = kept_e[j];
  } else {
    key_out[i] = PAD_KEY;
    e_out[i] = -1;
  }
}

struct ExplWorkspace {
  int32_t *counts, *offsets, *total, *num_kept;
  int32_t *e_row, *e_xfer, *e_next, *pos_of, *spos, *kept;
  uint32_t *e_parent, *pkey_in, *pkey_out;
  uint64_t *key_in, *key_out, *key2_in, *key2_out;
  int32_t *val_in, *val_out;
  int32_t *seg_begin, *seg_end, *match_p, *match_e, *hvals;
  unsigned long long* hkeys;
  uint8_t *keep, *taken_e;
  int64_t hmask;
  void* cub_tmp;
  size_t cub_bytes;
};

static size_t expl_layout(char* base, int64_t c, int64_t c_primary, int64_t n, int64_t parents,
                          ExplWorkspace* w) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> char* {
    char* p = base ? base + off : nullptr;
    off += align_up(bytes);
    return p;
  };
  const int64_t cc = c > 0 ? c : 1, nn = n > 0 ? n : 1, pp = parents > 0 ? parents : 1;
  int64_t h = 2;
  while (h < 2 * (c_primary > 0 ? c_primary : 1)) h <<= 1;
  w->hmask = h - 1;
  w->counts = (int32_t*)take(cc * 4);
  w->offsets = (int32_t*)take(cc * 4);
  w->total = (int32_t*)take(4);
  w->num_kept = (int32_t*)take(4);
  w->e_row = (int32_t*)take(nn * 4);
  w->e_xfer = (int32_t*)take(nn * 4);
  w->e_next = (int32_t*)take(nn * 4);
  w->pos_of = (int32_t*)take(nn * 4);
  w->spos = (int32_t*)take(nn * 4);
  w->kept = (int32_t*)take(nn * 4);
  w->e_parent = (uint32_t*)take(nn * 4);
  w->pkey_in = (uint32_t*)take(nn * 4);
  w->pkey_out = (uint32_t*)take(nn * 4);
  w->key_in = (uint64_t*)take(nn * 8);
  w->key_out = (uint64_t*)take(nn * 8);
  w->key2_in = (uint64_t*)take(nn * 8);
  w->key2_out = (uint64_t*)take(nn * 8);
  w->val_in = (int32_t*)take(nn * 4);
  w->val_out = (int32_t*)take(nn * 4);
  w->seg_begin = (int32_t*)take(2 * pp * 4);
  w->seg_end = (int32_t*)take(2 * pp * 4);
  w->match_p = (int32_t*)take(cc * 4);
  w->match_e = (int32_t*)take(cc * 4);
  w->hvals = (int32_t*)take(h * 4);
  w->hkeys = (unsigned long long*)take(h * 8);
  w->keep = (uint8_t*)take(nn);
  w->taken_e = (uint8_t*)take(nn);
  size_t need = 0, t = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, t, (int32_t*)nullptr, (int32_t*)nullptr, (int)cc);
  need = t > need ? t : need;
  cub::DeviceRadixSort::SortPairs(nullptr, t, (uint64_t*)nullptr, (uint64_t*)nullptr,
                                  (int32_t*)nullptr, (int32_t*)nullptr, (int)nn);
  need = t > need ? t : need;
  cub::DeviceRadixSort::SortPairs(nullptr, t, (uint32_t*)nullptr, (uint32_t*)nullptr,
                                  (int32_t*)nullptr, (int32_t*)nullptr, (int)nn);
  need = t > need ? t : need;
  cub::DeviceSelect::Flagged(nullptr, t, thrust::counting_iterator<int32_t>(0),
                             (uint8_t*)nullptr, (int32_t*)nullptr, (int32_t*)nullptr, (int)nn);
  need = t > need ? t : need;
  w->cub_bytes = need;
  w->cub_tmp = take(need);
  return off;
}

}  // namespace grs

extern "C" int64_t grs_proposals_exploration_workspace_bytes(int64_t num_candidates,
                                                             int64_t num_primary,
                                                             int64_t max_expanded,
                                                             int64_t num_parents) {
  ExplWorkspace w;
  return (int64_t)expl_layout(nullptr, num_candidates, num_primary, max_expanded, num_parents, &w);
}

extern "C" int grs_proposals_rank_exploration(
    const int64_t* batch_ids, const int64_t* sources, const int64_t* anchors,
    const float* probabilities, int64_t num_candidates, int64_t num_primary,
    const int64_t* parent_gate_counts, int64_t num_parents, const int32_t* xfer_offsets,
    const int32_t* xfer_counts, const int32_t* xfer_ids, const int32_t* gate_deltas,
    const int32_t* all_xfer_counts, int num_sources, int64_t max_expanded, int per_parent_cap,
    int exploration_per_parent, int64_t global_cap, int64_t* out_row, int64_t* out_xfer,
    int64_t* out_next_gate, int64_t* out_count, int64_t* out_metrics, void* workspace,
    int64_t workspace_bytes, int32_t* status, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t c = num_candidates, n = max_expanded, cp = num_primary;
  if (c < 0 || cp < 0 || cp > c || n < 0 || num_parents < 0 || per_parent_cap < 0 ||
      per_parent_cap > 0xfffe || exploration_per_parent < 0 || global_cap < 0 ||
      c > (1ll << 30) || n > (1ll << 30) || num_parents >= (1ll << 23))
    return GRS_ERR_SHAPE;
  ExplWorkspace w;
  const int64_t need = (int64_t)expl_layout((char*)workspace, c, cp, n, num_parents, &w);
  if (need > workspace_bytes) return GRS_ERR_WORKSPACE;
  cudaMemsetAsync(out_metrics, 0, 5 * sizeof(int64_t), s);
  if (c == 0 || n == 0 || num_parents == 0) {
    cudaMemsetAsync(out_count, 0, sizeof(int64_t), s);
    GRS_CUDA_CHECK_LAUNCH();
    return GRS_OK;
  }
  const int T = 256;
  prop_count_models_kernel<<<ceil_div(c, T), T, 0, counted(s)>>>(
      sources, c, cp, xfer_counts, all_xfer_counts, num_sources, w.counts, out_metrics, status);
  size_t tb = w.cub_bytes;
  cub::DeviceScan::ExclusiveSum(w.cub_tmp, tb, w.counts, w.offsets, (int)c, s);
  prop_total_kernel<<<1, 1, 0, counted(s)>>>(w.counts, w.offsets, c, w.total);
  prop_expand_kernel<<<ceil_div(c, T), T, 0, counted(s)>>>(
      batch_ids, sources, probabilities, c, w.counts, w.offsets, xfer_offsets, xfer_ids,
      gate_deltas, parent_gate_counts, num_parents, w.e_row, w.e_xfer, w.e_next, w.e_parent,
      w.key_in, w.val_in, n, status);
  prop_pad_kernel<<<ceil_div(n, T), T, 0, counted(s)>>>(w.total, n, w.key_in, w.val_in);
  // (next gate, probability desc, xfer), then stably by (parent, model)
  tb = w.cub_bytes;
  cub::DeviceRadixSort::SortPairs(w.cub_tmp, tb, w.key_in, w.key_out, w.val_in, w.val_out,
                                  (int)n, 0, 64, s);
  prop_model_key_kernel<<<ceil_div(n, T), T, 0, counted(s)>>>(w.val_out, n, w.total, w.e_parent,
                                                             w.e_row, cp, w.pkey_in);
  tb = w.cub_bytes;
  cub::DeviceRadixSort::SortPairs(w.cub_tmp, tb, w.pkey_in, w.pkey_out, w.val_out, w.val_in,
                                  (int)n, 0, 32, s);
  cudaMemsetAsync(w.seg_begin, 0, 2 * num_parents * sizeof(int32_t), s);
  cudaMemsetAsync(w.seg_end, 0, 2 * num_parents * sizeof(int32_t), s);
  prop_positions_kernel<<<ceil_div(n, T), T, 0, counted(s)>>>(w.pkey_out, w.val_in, n, w.pos_of,
                                                             w.seg_begin, w.seg_end);
  // pair the two models' candidates on (parent, source, anchor)
  cudaMemsetAsync(w.hkeys, 0, (w.hmask + 1) * sizeof(unsigned long long), s);
  if (cp > 0)
    prop_join_insert_kernel<<<ceil_div(cp, T), T, 0, counted(s)>>>(
        batch_ids, sources, anchors, cp, w.hkeys, w.hvals, w.hmask, w.match_e, status);
  if (c > cp)
    prop_join_lookup_kernel<<<ceil_div(c - cp, T), T, 0, counted(s)>>>(
        batch_ids, sources, anchors, cp, c, w.hkeys, w.hvals, w.hmask, w.match_p, w.match_e);
  cudaMemsetAsync(w.keep, 0, n, s);
  cudaMemsetAsync(w.taken_e, 0, n, s);
  prop_select_exploration_kernel<<<(unsigned)num_parents, EXPL_THREADS, 0, counted(s)>>>(
      w.val_in, w.pos_of, w.seg_begin, w.seg_end, w.e_row, w.offsets, cp, w.match_p, w.match_e,
      per_parent_cap, exploration_per_parent, w.keep, w.taken_e, w.spos, out_metrics);
  tb = w.cub_bytes;
  cub::DeviceSelect::Flagged(w.cub_tmp, tb, thrust::counting_iterator<int32_t>(0), w.keep,
                             w.kept, w.num_kept, (int)n, s);
  prop_exploration_keys_kernel<<<ceil_div(n, T), T, 0, counted(s)>>>(
      w.kept, w.num_kept, n, w.e_next, w.e_row, w.e_xfer, w.e_parent, w.spos, probabilities,
      parent_gate_counts, w.key2_in, w.key_in, w.val_in, status);
  // LSD: the tie order first, then the ranking key (both sorts stable)
  tb = w.cub_bytes;
  cub::DeviceRadixSort::SortPairs(w.cub_tmp, tb, w.key2_in, w.key2_out, w.val_in, w.val_out,
                                  (int)n, 0, 64, s);
  prop_gather_keys_kernel<<<ceil_div(n, T), T, 0, counted(s)>>>(w.val_out, n, w.kept, w.num_kept,
                                                               w.key_in, w.key_out, w.val_in);
  tb = w.cub_bytes;
  cub::DeviceRadixSort::SortPairs(w.cub_tmp, tb, w.key_out, w.key_in, w.val_in, w.val_out,
                                  (int)n, 0, 64, s);
  if (global_cap > 0)
    prop_output_kernel<<<ceil_div(global_cap, T), T, 0, counted(s)>>>(
        w.val_out, w.num_kept, global_cap, w.e_row, w.e_xfer, w.e_next, out_row, out_xfer,
        out_next_gate, out_count);
  else
    cudaMemsetAsync(out_count, 0, sizeof(int64_t), s);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}
