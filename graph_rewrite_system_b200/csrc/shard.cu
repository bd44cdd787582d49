// Ranked-record exchange of the beam search sharded over the GPUs of a node.
//
// The single-GPU search (paged_rollout_benchmark.py:898-1207) ranks every
// proposal of the level globally - next gate count ascending, probability
// descending, parent gate count ascending, then expansion order (:967-1005) -
// and walks that list in its accept loop (:1013-1046).  Sharded, each GPU
// ranks its own beams' proposals; these kernels turn the per-GPU ranked lists
// into the global list and route the accepted children:
//
//   shard_records_kernel  packs this GPU's ranked list into records whose two
//                         keys order like the global ranking (field-major
//                         [KEY1 | KEY2 | FP | AUX] x width, then 4 metrics);
//   shard_count_kernel +  merge the gathered, individually sorted lists by
//   shard_merge_kernel    rank (a merge-path position from binary searches in
//                         the other lists) straight into the arrays the
//                         accept loop reads;
//   shard_route_kernel    places the accepted children on GPUs (each GPU keeps
//                         its own children up to an even share, the overflow
//                         goes in order to the GPUs with room, lowest first)
//                         and writes this GPU's keep / send / receive lists.
//
// Record keys: KEY1 = next_gate << 44 | ~prob_bits << 12 | parent_gate and
// KEY2 = global_parent << 27 | xfer << 11 | candidate row within the parent.
// AUX = child_next_slot | valid << 32.  Padding rows have KEY1 = ABSENT.
#include "grs_common.cuh"
#include "topology_table.cuh"

namespace grs {

constexpr int64_t REC_ABSENT = 0x7fffffffffffffffll;
constexpr int REC_FIELDS = 4, REC_METRICS = 4;
constexpr int SHARD_MAX_WORLD = 64;

__device__ __forceinline__ bool rec_less(int64_t a1, int64_t a2, int64_t b1, int64_t b2) {
  return a1 < b1 || (a1 == b1 && a2 < b2);
}

__global__ void shard_records_kernel(int64_t width, const int64_t* count, const int64_t* rows,
                                     const int64_t* xfers, const int64_t* next_gate,
                                     const float* probs, const int64_t* cand_batch, int64_t k,
                                     const int64_t* gate, const int64_t* global_index,
                                     const int32_t* next_slot, const int32_t* table,
                                     const uint8_t* valid, const int64_t* fp,
                                     const int64_t* ranked_metrics, const int32_t* free_count,
                                     int64_t capacity, int64_t* out, int32_t* status) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t n = *count;
  if (j == 0) {
    int64_t* m = out + REC_FIELDS * width;
    m[0] = n;
    m[1] = ranked_metrics ? ranked_metrics[0] : 0;
    m[2] = ranked_metrics ? ranked_metrics[1] : 0;
    m[3] = free_count ? capacity - *free_count : 0;
  }
  if (j >= width) return;
  int64_t key1 = REC_ABSENT, key2 = 0, f = 0, aux = 0;
  if (j < n) {
    const int64_t row = rows[j];
    const int64_t parent = cand_batch[row];
    const int64_t x = xfers[j];
    const int64_t ng = next_gate[j], pg = gate[parent], gp = global_index[parent];
    const int64_t cand = row % k;
    if (ng < 0 || ng >= 4096 || pg < 0 || pg >= 4096 || gp < 0 || gp >= (1ll << 23) || x < 0 ||
        x >= 65536 || cand >= 2048) {
      set_status(status, GRS_ERR_TOO_LARGE);  // a field overflows its key bits
    } else {
      const uint32_t bits = __float_as_uint(probs[row]);
      key1 = (ng << 44) | ((int64_t)(0xffffffffu - bits) << 12) | pg;
      key2 = (gp << 27) | (x << 11) | cand;
      f = fp[j];
      const int64_t child_next = (int64_t)next_slot[parent] + table[x * TAB_WIDTH + TAB_DST_LEN];
      aux = child_next | ((int64_t)(valid[j] != 0) << 32);
    }
  }
  out[j] = key1;
  out[width + j] = key2;
  out[2 * width + j] = f;
  out[3 * width + j] = aux;
}

// One warp: per-list present counts (the ABSENT rows sit at the end of every
// list), the merged count and the summed metrics.
__global__ void shard_count_kernel(const int64_t* gathered, int world, int64_t width,
                                   int64_t stride, int64_t cap, int64_t* count,
                                   int64_t* metrics) {
  __shared__ unsigned long long total;
  const int t = threadIdx.x;
  if (t == 0) total = 0;
  __syncthreads();
  for (int q = t; q < world; q += blockDim.x) {
    const int64_t* k1 = gathered + q * stride;
    int64_t lo = 0, hi = width;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (k1[mid] != REC_ABSENT) lo = mid + 1; else hi = mid;
    }
    atomicAdd(&total, (unsigned long long)lo);
  }
  for (int m = t; m < REC_METRICS; m += blockDim.x) {
    int64_t s = 0;
    for (int q = 0; q < world; ++q) s += gathered[q * stride + REC_FIELDS * width + m];
    metrics[m] = s;
  }
  __syncthreads();
  if (t == 0) *count = min((int64_t)total, cap);
}

// Records of list q ordered before (a1, a2); ties (which distinct proposals
// never produce) count as before when `inclusive`, so equal keys keep list
// order and every position stays distinct.
__device__ __forceinline__ int64_t records_before(const int64_t* k1, const int64_t* k2,
                                                  int64_t n, int64_t a1, int64_t a2,
                                                  bool inclusive) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    const int64_t b1 = k1[mid];
    const bool before = b1 < a1 || (b1 == a1 && (inclusive ? k2[mid] <= a2 : k2[mid] < a2));
    if (before) lo = mid + 1; else hi = mid;
  }
  return lo;
}

__global__ void shard_merge_kernel(const int64_t* gathered, int world, int64_t width,
                                   int64_t stride, int64_t cap, const int64_t* count,
                                   uint8_t* valid, int64_t* fp, int64_t* next_gate, int64_t* src,
                                   int64_t* index, int64_t* child_next, int32_t* status) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < cap && t >= *count) {  // padding past the merged count
    valid[t] = 0;
    fp[t] = 0;
    next_gate[t] = 0;
    src[t] = world;
    index[t] = 0;
    child_next[t] = 0;
  }
  if (t >= (int64_t)world * width) return;
  const int r = (int)(t / width);
  const int64_t j = t - (int64_t)r * width;
  const int64_t* base = gathered + r * stride;
  const int64_t a1 = base[j], a2 = base[width + j];
  if (j + 1 < width) {  // every list must arrive sorted, padding last
    const int64_t b1 = base[j + 1], b2 = base[width + j + 1];
    if (a1 == REC_ABSENT ? b1 != REC_ABSENT : (b1 != REC_ABSENT && !rec_less(a1, a2, b1, b2)))
      set_status(status, GRS_ERR_ORDER);
  }
  if (a1 == REC_ABSENT) return;
  int64_t p = j;
  for (int q = 0; q < world; ++q) {
    if (q == r) continue;
    const int64_t* other = gathered + q * stride;
    p += records_before(other, other + width, width, a1, a2, q < r);
  }
  if (p >= cap) return;
  const int64_t aux = base[3 * width + j];
  valid[p] = (uint8_t)((aux >> 32) & 1);
  fp[p] = base[2 * width + j];
  next_gate[p] = a1 >> 44;
  src[p] = r;
  index[p] = j;
  child_next[p] = aux & 0xffffffffll;
}

// Stable rank of every element of a 1024-wide chunk among the elements with
// the same key (keys in [0, nkeys), -1 = not counted), continuing the running
// per-key totals of earlier chunks.  All threads of the block call it.
constexpr int ROUTE_THREADS = 1024, ROUTE_WARPS = ROUTE_THREADS / 32,
              ROUTE_KEYS = SHARD_MAX_WORLD + 1;
__device__ int chunk_key_rank(int key, int nkeys, int* warp_counts, int* running) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned peers = __match_any_sync(0xffffffffu, key);
  for (int q = lane; q < nkeys; q += 32) warp_counts[warp * ROUTE_KEYS + q] = 0;
  __syncwarp();
  if (key >= 0 && lane == __ffs(peers) - 1) warp_counts[warp * ROUTE_KEYS + key] = __popc(peers);
  __syncthreads();
  int r = -1;
  if (key >= 0) {
    r = running[key] + __popc(peers & ((1u << lane) - 1u));
    for (int w = 0; w < warp; ++w) r += warp_counts[w * ROUTE_KEYS + key];
  }
  __syncthreads();
  if (tid < nkeys) {
    int s = 0;
    for (int w = 0; w < ROUTE_WARPS; ++w) s += warp_counts[w * ROUTE_KEYS + tid];
    running[tid] += s;
  }
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(ROUTE_THREADS) shard_route_kernel(
    const int64_t* child_proposal, const int64_t* summary, const int64_t* src,
    const int64_t* index, const int64_t* child_next, int64_t cap, int beam_size, int world,
    int me, int64_t* pairs, int64_t* extent, int64_t* keep_local, int64_t* keep_global,
    int64_t* out_local, int64_t* in_global, int32_t* status) {
  extern __shared__ unsigned char route_smem[];
  uint16_t* pos = reinterpret_cast<uint16_t*>(route_smem);                 // [beam_size]
  uint8_t* csrc = reinterpret_cast<uint8_t*>(pos + beam_size);              // [beam_size]
  uint8_t* cdst = csrc + beam_size;                                         // [beam_size]
  __shared__ int warp_counts[ROUTE_WARPS * ROUTE_KEYS];
  __shared__ int running[ROUTE_KEYS];
  __shared__ int quota[SHARD_MAX_WORLD], room_end[SHARD_MAX_WORLD], in_base[SHARD_MAX_WORLD];
  __shared__ int pair_count[SHARD_MAX_WORLD * SHARD_MAX_WORLD];
  __shared__ unsigned long long s_extent;
  const int tid = threadIdx.x;
  const int a = (int)min(max(summary[0], (int64_t)0), (int64_t)beam_size);
  for (int q = tid; q < ROUTE_KEYS; q += ROUTE_THREADS) running[q] = 0;
  for (int q = tid; q < world * world; q += ROUTE_THREADS) pair_count[q] = 0;
  if (tid == 0) s_extent = 0;
  __syncthreads();
  // 1. position of every child among the children of the same source GPU
  for (int base = 0; base < a; base += ROUTE_THREADS) {
    const int j = base + tid;
    int key = -1;
    if (j < a) {
      const int64_t p = child_proposal[j];
      const int64_t s = (p >= 0 && p < cap) ? src[p] : -1;
      if (s < 0 || s >= world) {
        set_status(status, GRS_ERR_ORDER);
        csrc[j] = 0xff;
      } else {
        key = (int)s;
        csrc[j] = (uint8_t)s;
        atomicMax(&s_extent, (unsigned long long)max(child_next[p], (int64_t)0));
      }
    }
    const int r = chunk_key_rank(key, world, warp_counts, running);
    if (key >= 0) pos[j] = (uint16_t)r;
  }
  // 2. quotas, kept counts and the room left on every GPU (prefix)
  if (tid == 0) {
    int end = 0;
    for (int q = 0; q < world; ++q) {
      quota[q] = a / world + (q < a % world ? 1 : 0);
      end += quota[q] - min(running[q], quota[q]);
      room_end[q] = end;
    }
  }
  __syncthreads();
  for (int q = tid; q < ROUTE_KEYS; q += ROUTE_THREADS) running[q] = 0;
  __syncthreads();
  // 3. destinations: kept at home, overflow in order to the GPUs with room
  for (int base = 0; base < a; base += ROUTE_THREADS) {
    const int j = base + tid;
    const bool real = j < a && csrc[j] < world;
    const int s = real ? csrc[j] : 0;
    const bool over = real && pos[j] >= quota[s];
    const int o = chunk_key_rank(over ? 0 : -1, 1, warp_counts, running);
    if (real) {
      int d = s;
      if (over) {
        d = -1;
        for (int q = 0; q < world; ++q)
          if (room_end[q] > o) { d = q; break; }
        if (d < 0) { set_status(status, GRS_ERR_ORDER); d = s; }
      }
      cdst[j] = (uint8_t)d;
      atomicAdd(&pair_count[s * world + d], 1);
      if (s == me) {
        const int64_t li = index[child_proposal[j]];
        if (d == me) {
          keep_local[pos[j]] = li;
          keep_global[pos[j]] = j;
        } else {
          out_local[pos[j] - quota[me]] = li;
        }
      }
    } else if (j < a) {
      cdst[j] = 0xff;
    }
  }
  __syncthreads();
  if (tid == 0) {
    int b = 0;
    for (int q = 0; q < world; ++q) {
      in_base[q] = b;
      if (q != me) b += pair_count[q * world + me];
    }
  }
  for (int q = tid; q < ROUTE_KEYS; q += ROUTE_THREADS) running[q] = 0;
  __syncthreads();
  // 4. children arriving here, grouped by source GPU in global order
  for (int base = 0; base < a; base += ROUTE_THREADS) {
    const int j = base + tid;
    int key = -1;
    if (j < a && cdst[j] == me && csrc[j] != me) key = csrc[j];
    const int r = chunk_key_rank(key, world, warp_counts, running);
    if (key >= 0) in_global[in_base[key] + r] = j;
  }
  for (int q = tid; q < world * world; q += ROUTE_THREADS) pairs[q] = pair_count[q];
  if (tid == 0) *extent = (int64_t)s_extent;
}


// ---- multi-segment row copies ------------------------------------------------
// A segment copies `units` units of `unit_bytes` per row from src to dst.  Unit
// k of row i sits at base + index[i * units + k] * unit_stride when the side
// has an index, else at base + i * row_stride + k * unit_stride.  One launch
// packs every field of the rows that change GPU into contiguous send rows,
// unpacks received rows into the field tensors and cache pages, or reorders a
// beam.
constexpr int ROWS_MAX_SEGMENTS = 40, ROWS_SEG_WORDS = 10;
struct RowSegment {
  const uint8_t* src; int64_t src_row, src_unit; const int64_t* src_index;
  uint8_t* dst; int64_t dst_row, dst_unit; const int64_t* dst_index;
  int64_t unit_bytes, units;
};
struct RowSegments { RowSegment seg[ROWS_MAX_SEGMENTS]; int n; };

template <typename V>
__device__ __forceinline__ void copy_unit(const uint8_t* s, uint8_t* d, int64_t bytes) {
  const V* sv = reinterpret_cast<const V*>(s);
  V* dv = reinterpret_cast<V*>(d);
  for (int64_t e = threadIdx.x; e < bytes / (int64_t)sizeof(V); e += blockDim.x) dv[e] = sv[e];
}

__global__ void __launch_bounds__(256) rows_copy_kernel(RowSegments segs, const int64_t* n_dev,
                                                        int64_t n_max) {
  // work items: (segment, row, unit), segment-major
  __shared__ int64_t start[ROWS_MAX_SEGMENTS + 1];
  if (threadIdx.x == 0) {
    const int64_t rows = n_dev ? max((int64_t)0, min(*n_dev, n_max)) : n_max;
    start[0] = 0;
    for (int g = 0; g < segs.n; ++g) start[g + 1] = start[g] + rows * segs.seg[g].units;
  }
  __syncthreads();
  const int64_t items = start[segs.n];
  for (int64_t w = blockIdx.x; w < items; w += gridDim.x) {
    int g = 0;
    while (w >= start[g + 1]) ++g;
    const RowSegment& sg = segs.seg[g];
    const int64_t local = w - start[g];
    const int64_t i = local / sg.units, k = local - i * sg.units;
    const uint8_t* src = sg.src + (sg.src_index ? sg.src_index[local] * sg.src_unit
                                                : i * sg.src_row + k * sg.src_unit);
    uint8_t* dst = sg.dst + (sg.dst_index ? sg.dst_index[local] * sg.dst_unit
                                          : i * sg.dst_row + k * sg.dst_unit);
    const uint64_t align = (uint64_t)src | (uint64_t)dst | (uint64_t)sg.unit_bytes;
    if ((align & 15) == 0) copy_unit<uint4>(src, dst, sg.unit_bytes);
    else if ((align & 7) == 0) copy_unit<uint2>(src, dst, sg.unit_bytes);
    else if ((align & 3) == 0) copy_unit<uint32_t>(src, dst, sg.unit_bytes);
    else copy_unit<uint8_t>(src, dst, sg.unit_bytes);
  }
}

}  // namespace grs

using namespace grs;

extern "C" int grs_shard_records(int64_t width, const int64_t* count, const int64_t* rows,
                                 const int64_t* xfers, const int64_t* next_gate,
                                 const float* probs, const int64_t* cand_batch, int64_t k,
                                 const int64_t* gate, const int64_t* global_index,
                                 const int32_t* next_slot, const int32_t* table,
                                 const uint8_t* valid, const int64_t* fp,
                                 const int64_t* ranked_metrics, const int32_t* free_count,
                                 int64_t capacity, int64_t* out, int32_t* status, void* stream) {
  if (width < 0 || k <= 0 || count == nullptr || out == nullptr) return GRS_ERR_SHAPE;
  const int64_t threads = width > 0 ? width : 1;
  shard_records_kernel<<<ceil_div(threads, 256), 256, 0, counted((cudaStream_t)stream)>>>(
      width, count, rows, xfers, next_gate, probs, cand_batch, k, gate, global_index, next_slot,
      table, valid, fp, ranked_metrics, free_count, capacity, out, status);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_shard_merge(const int64_t* gathered, int world, int64_t width, int64_t stride,
                               int64_t cap, int64_t* count, int64_t* metrics, uint8_t* valid,
                               int64_t* fp, int64_t* next_gate, int64_t* src, int64_t* index,
                               int64_t* child_next, int32_t* status, void* stream) {
  if (world < 1 || world > SHARD_MAX_WORLD || width < 0 || cap < 0 ||
      stride < REC_FIELDS * width + REC_METRICS || cap > (int64_t)world * width)
    return GRS_ERR_SHAPE;
  cudaStream_t s = (cudaStream_t)stream;
  shard_count_kernel<<<1, 64, 0, counted(s)>>>(gathered, world, width, stride, cap, count,
                                               metrics);
  const int64_t n = max((int64_t)world * width, cap);
  if (n > 0)
    shard_merge_kernel<<<ceil_div(n, 256), 256, 0, counted(s)>>>(
        gathered, world, width, stride, cap, count, valid, fp, next_gate, src, index, child_next,
        status);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_shard_route(const int64_t* child_proposal, const int64_t* summary,
                               const int64_t* src, const int64_t* index,
                               const int64_t* child_next, int64_t cap, int beam_size, int world,
                               int me, int64_t* pairs, int64_t* extent, int64_t* keep_local,
                               int64_t* keep_global, int64_t* out_local, int64_t* in_global,
                               int32_t* status, void* stream) {
  if (world < 1 || world > SHARD_MAX_WORLD || me < 0 || me >= world || beam_size < 0 ||
      beam_size > 8192)
    return GRS_ERR_SHAPE;
  const size_t smem = (size_t)beam_size * 4;  // uint16 position + uint8 source + uint8 dest
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(shard_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         8192 * 4);
    attr[dev] = true;
  }
  shard_route_kernel<<<1, ROUTE_THREADS, smem, counted((cudaStream_t)stream)>>>(
      child_proposal, summary, src, index, child_next, cap, beam_size, world, me, pairs, extent,
      keep_local, keep_global, out_local, in_global, status);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_rows_copy(int nseg, const int64_t* segments, const int64_t* n_dev,
                             int64_t n_max, void* stream) {
  if (nseg < 0 || nseg > ROWS_MAX_SEGMENTS || n_max < 0 || (nseg > 0 && segments == nullptr))
    return GRS_ERR_SHAPE;
  RowSegments p{};
  p.n = nseg;
  for (int g = 0; g < nseg; ++g) {
    const int64_t* w = segments + g * ROWS_SEG_WORDS;
    RowSegment& sg = p.seg[g];
    sg.src = reinterpret_cast<const uint8_t*>(w[0]);
    sg.src_row = w[1]; sg.src_unit = w[2];
    sg.src_index = reinterpret_cast<const int64_t*>(w[3]);
    sg.dst = reinterpret_cast<uint8_t*>(w[4]);
    sg.dst_row = w[5]; sg.dst_unit = w[6];
    sg.dst_index = reinterpret_cast<const int64_t*>(w[7]);
    sg.unit_bytes = w[8]; sg.units = w[9];
    if (sg.unit_bytes < 0 || sg.units < 1 || (sg.unit_bytes > 0 && (!sg.src || !sg.dst)))
      return GRS_ERR_SHAPE;
  }
  if (nseg == 0 || n_max == 0) return GRS_OK;
  int64_t work = 0;
  for (int g = 0; g < nseg; ++g) work += n_max * p.seg[g].units;
  const int blocks = (int)(work < 148 * 8 ? work : 148 * 8);
  rows_copy_kernel<<<blocks, 256, 0, counted((cudaStream_t)stream)>>>(p, n_dev, n_max);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}
