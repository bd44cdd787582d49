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
  prop_count_kernel<<<ceil_div(c, T), T, 0, s>>>(sources, c, xfer_counts, all_xfer_counts,
                                                 num_sources, w.counts, out_metrics, status);
  size_t tb = w.cub_bytes;
  cub::DeviceScan::ExclusiveSum(w.cub_tmp, tb, w.counts, w.offsets, (int)c, s);
  prop_total_kernel<<<1, 1, 0, s>>>(w.counts, w.offsets, c, w.total);
  prop_expand_kernel<<<ceil_div(c, T), T, 0, s>>>(
      batch_ids, sources, probabilities, c, w.counts, w.offsets, xfer_offsets, xfer_ids,
      gate_deltas, parent_gate_counts, num_parents, w.e_row, w.e_xfer, w.e_next, w.e_parent,
      w.key_in, w.val_in, n, status);
  prop_pad_kernel<<<ceil_div(n, T), T, 0, s>>>(w.total, n, w.key_in, w.val_in);
  // (next_gate, prob desc, xfer) then stable by parent.
  tb = w.cub_bytes;
  cub::DeviceRadixSort::SortPairs(w.cub_tmp, tb, w.key_in, w.key_out, w.val_in, w.val_out,
                                  (int)n, 0, 64, s);
  prop_parent_key_kernel<<<ceil_div(n, T), T, 0, s>>>(w.val_out, n, w.total, w.e_parent,
                                                      w.pkey_in);
  tb = w.cub_bytes;
  cub::DeviceRadixSort::SortPairs(w.cub_tmp, tb, w.pkey_in, w.pkey_out, w.val_out, w.val_in,
                                  (int)n, 0, 32, s);
  prop_segment_start_kernel<<<ceil_div(n, T), T, 0, s>>>(w.pkey_out, n, w.seg_start);
  tb = w.cub_bytes;
  cub::DeviceScan::InclusiveScan(w.cub_tmp, tb, w.seg_start, w.val_out, cub::Max(), (int)n, s);
  prop_flag_kernel<<<ceil_div(n, T), T, 0, s>>>(w.pkey_out, w.val_out, n, per_parent_cap,
                                                w.flags);
  tb = w.cub_bytes;
  cub::DeviceSelect::Flagged(w.cub_tmp, tb, w.val_in, w.flags, w.kept, w.num_kept, (int)n, s);
  prop_global_key_kernel<<<ceil_div(n, T), T, 0, s>>>(w.kept, w.num_kept, n, w.e_next, w.e_row,
                                                      w.e_parent, probabilities,
                                                      parent_gate_counts, w.key_in, w.val_in,
                                                      status);
  tb = w.cub_bytes;
  cub::DeviceRadixSort::SortPairs(w.cub_tmp, tb, w.key_in, w.key_out, w.val_in, w.val_out,
                                  (int)n, 0, 64, s);
  if (global_cap > 0)
    prop_output_kernel<<<ceil_div(global_cap, T), T, 0, s>>>(
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
