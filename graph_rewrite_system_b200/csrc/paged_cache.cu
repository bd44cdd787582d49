// PagedKVCache fork / copy-on-write / append / release, in place on device
// arenas (reference paged_cache.py:16-238).
//
// Allocation is bit-exact with the reference's sequential host loop: the
// free list is a device array whose top is free_list[free_count - 1]; parent
// i of an append batch takes free_list[free_count - 1 - i] (retains never
// touch the free list and nothing is released inside append_batch,
// paged_cache.py:140-181).  Release appends the pages that reach refcount 0
// in the order of the decrement that zeroed them in the (handle, block) scan
// (paged_cache.py:99-105): that decrement is the page's last one in scan
// order, found with an atomicMax over scan positions, and a single-CTA ordered
// compaction appends the pages.
#include "grs_common.cuh"

namespace grs {

struct CacheArenas {
  void* keys; void* values;           // [L, capacity, page, H, D]
  void* actions;                      // [capacity, page, W]
  void* rkeys; void* rvalues;         // [capacity, page, H, D] (nullable)
  int layers, capacity, page, hd, width, elem;  // hd = H * D; elem = bytes per element
};

__device__ __forceinline__ int blocks_for(int length, int page) { return (length + page - 1) / page; }

// One thread per parent: retain shared pages, allocate the child page, write
// the child block-table row and length.
__global__ void cache_fork_kernel(int32_t* __restrict__ refcounts,
                                  const int32_t* __restrict__ free_list,
                                  const int32_t* __restrict__ free_count, int capacity,
                                  const int32_t* __restrict__ ptable, int64_t pstride,
                                  const int32_t* __restrict__ plengths, int n, int page,
                                  int32_t* __restrict__ ctable, int64_t cstride,
                                  int32_t* __restrict__ clengths, int ccols,
                                  int32_t* __restrict__ status) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int len = plengths[i];
  const int nb = blocks_for(len, page);
  const int offset = len % page;
  const int keep = offset == 0 ? nb : nb - 1;  // pages shared with the child
  const int32_t* prow = ptable + (int64_t)i * pstride;
  int32_t* crow = ctable + (int64_t)i * cstride;
  if (keep + 1 > ccols) { set_status(status, GRS_ERR_SHAPE); return; }
  // Error paths record a status and write page 0 so that no table ever holds
  // an out-of-range page id.
  for (int j = 0; j < keep; ++j) {
    const int p = prow[j];
    if (p < 0 || p >= capacity) {
      set_status(status, GRS_ERR_BAD_PAGE);
      crow[j] = 0;
      continue;
    }
    // children of one parent (and siblings sharing ancestors) retain the
    // same pages: one atomic per distinct page among the active lanes
    const unsigned active = __activemask();
    const unsigned peers = __match_any_sync(active, p);
    if ((threadIdx.x & 31) == __ffs(peers) - 1) {
      const int old = atomicAdd(&refcounts[p], __popc(peers));
      if (old <= 0) set_status(status, GRS_ERR_BAD_PAGE);
    }
    crow[j] = p;
  }
  const int fc = *free_count;
  int page_id = 0;
  if (i >= fc) {
    set_status(status, GRS_ERR_EXHAUSTED);
  } else {
    const int candidate = free_list[fc - 1 - i];
    if (candidate < 0 || candidate >= capacity || refcounts[candidate] != 0) {
      set_status(status, GRS_ERR_CORRUPT);
    } else {
      page_id = candidate;
      refcounts[page_id] = 1;
    }
  }
  crow[keep] = page_id;
  for (int j = keep + 1; j < ccols; ++j) crow[j] = 0;
  clengths[i] = len + 1;
}

// Copy `rows` rows of `row_bytes` bytes from page src to page dst within one
// arena segment (16-byte vectors when aligned, else 4-byte words).
__device__ __forceinline__ void copy_rows(char* base, int64_t page_bytes, int src, int dst,
                                          int rows, int64_t row_bytes) {
  const int64_t bytes = (int64_t)rows * row_bytes;
  const char* s = base + (int64_t)src * page_bytes;
  char* d = base + (int64_t)dst * page_bytes;
  if ((page_bytes & 15) == 0 && ((uintptr_t)base & 15) == 0 && (bytes & 15) == 0) {
    for (int64_t v = threadIdx.x; v < bytes / 16; v += blockDim.x)
      reinterpret_cast<uint4*>(d)[v] = reinterpret_cast<const uint4*>(s)[v];
  } else {
    for (int64_t v = threadIdx.x; v < bytes / 4; v += blockDim.x)
      reinterpret_cast<uint32_t*>(d)[v] = reinterpret_cast<const uint32_t*>(s)[v];
  }
}

__device__ __forceinline__ void write_row(char* base, int64_t page_bytes, int64_t row_bytes,
                                          int page_id, int offset, const char* src) {
  char* d = base + (int64_t)page_id * page_bytes + (int64_t)offset * row_bytes;
  if ((row_bytes & 15) == 0 && ((uintptr_t)d & 15) == 0 && ((uintptr_t)src & 15) == 0) {
    for (int64_t v = threadIdx.x; v < row_bytes / 16; v += blockDim.x)
      reinterpret_cast<uint4*>(d)[v] = reinterpret_cast<const uint4*>(src)[v];
  } else {
    for (int64_t v = threadIdx.x; v < row_bytes / 4; v += blockDim.x)
      reinterpret_cast<uint32_t*>(d)[v] = reinterpret_cast<const uint32_t*>(src)[v];
  }
}

// One CTA per child: COW-copy the valid rows of the parent's partial tail
// page into the child page in every arena, then write the new row.
__global__ void cache_write_kernel(CacheArenas ar, const int32_t* __restrict__ ptable,
                                   int64_t pstride, const int32_t* __restrict__ plengths,
                                   const int32_t* __restrict__ ctable, int64_t cstride, int n,
                                   const char* __restrict__ new_keys,
                                   const char* __restrict__ new_values,
                                   const char* __restrict__ new_actions,
                                   const char* __restrict__ new_rkeys,
                                   const char* __restrict__ new_rvalues,
                                   int32_t* __restrict__ free_count,
                                   const int32_t* __restrict__ status) {
  const int i = blockIdx.x;
  if (i == 0 && threadIdx.x == 0) {
    const int fc = *free_count;
    *free_count = fc >= n ? fc - n : 0;
  }
  if (*status != 0) return;
  const int len = plengths[i];
  const int offset = len % ar.page;
  const int nb = blocks_for(len, ar.page);
  const int dst = ctable[(int64_t)i * cstride + (offset == 0 ? nb : nb - 1)];
  if (dst < 0 || dst >= ar.capacity) return;
  const int64_t kv_row = (int64_t)ar.hd * ar.elem;
  const int64_t kv_page = kv_row * ar.page;
  const int64_t kv_layer = kv_page * ar.capacity;
  const int64_t act_row = (int64_t)ar.width * ar.elem;
  const int64_t act_page = act_row * ar.page;
  if (offset != 0) {
    const int src = ptable[(int64_t)i * pstride + nb - 1];
    if (src < 0 || src >= ar.capacity) return;
    for (int l = 0; l < ar.layers; ++l) {
      copy_rows((char*)ar.keys + l * kv_layer, kv_page, src, dst, offset, kv_row);
      copy_rows((char*)ar.values + l * kv_layer, kv_page, src, dst, offset, kv_row);
    }
    copy_rows((char*)ar.actions, act_page, src, dst, offset, act_row);
    if (new_rkeys) {
      copy_rows((char*)ar.rkeys, kv_page, src, dst, offset, kv_row);
      copy_rows((char*)ar.rvalues, kv_page, src, dst, offset, kv_row);
    }
  }
  for (int l = 0; l < ar.layers; ++l) {
    const int64_t in_off = ((int64_t)l * n + i) * kv_row;
    write_row((char*)ar.keys + l * kv_layer, kv_page, kv_row, dst, offset, new_keys + in_off);
    write_row((char*)ar.values + l * kv_layer, kv_page, kv_row, dst, offset, new_values + in_off);
  }
  write_row((char*)ar.actions, act_page, act_row, dst, offset, new_actions + (int64_t)i * act_row);
  if (new_rkeys) {
    write_row((char*)ar.rkeys, kv_page, kv_row, dst, offset, new_rkeys + (int64_t)i * kv_row);
    write_row((char*)ar.rvalues, kv_page, kv_row, dst, offset, new_rvalues + (int64_t)i * kv_row);
  }
}

// The same as cache_write_kernel when every row is a whole number of 16-byte
// vectors and every base is 16-byte aligned (the layouts the model uses):
// one CTA per child treats its segments (K and V of each layer, actions,
// readout K and V) as one flat list of 16-byte vectors - the COW rows of the
// parent's tail page, then the new row - and moves WV_BATCH of them per
// thread per round, all loads before the stores, so each round costs one
// memory latency instead of one per vector.
constexpr int WV_THREADS = 256;
constexpr int WV_BATCH = 8;
__global__ void __launch_bounds__(WV_THREADS) cache_write_vec_kernel(
    CacheArenas ar, const int32_t* __restrict__ ptable, int64_t pstride,
    const int32_t* __restrict__ plengths, const int32_t* __restrict__ ctable, int64_t cstride,
    int n, const char* __restrict__ new_keys, const char* __restrict__ new_values,
    const char* __restrict__ new_actions, const char* __restrict__ new_rkeys,
    const char* __restrict__ new_rvalues, int32_t* __restrict__ free_count,
    const int32_t* __restrict__ status) {
  const int i = blockIdx.x;
  if (i == 0 && threadIdx.x == 0) {
    const int fc = *free_count;
    *free_count = fc >= n ? fc - n : 0;
  }
  if (*status != 0) return;
  const int len = plengths[i];
  const int offset = len % ar.page;
  const int nb = blocks_for(len, ar.page);
  const int dst = ctable[(int64_t)i * cstride + (offset == 0 ? nb : nb - 1)];
  if (dst < 0 || dst >= ar.capacity) return;
  int src = dst;
  if (offset != 0) {
    src = ptable[(int64_t)i * pstride + nb - 1];
    if (src < 0 || src >= ar.capacity) return;
  }
  const int rows = offset + 1;                       // COW rows, then the new row
  const int kv_vecs = ar.hd * ar.elem / 16, act_vecs = ar.width * ar.elem / 16;
  const int64_t kv_row = (int64_t)ar.hd * ar.elem, act_row = (int64_t)ar.width * ar.elem;
  const int64_t kv_page = kv_row * ar.page, act_page = act_row * ar.page;
  const int64_t kv_layer = kv_page * ar.capacity;
  const int per_kv = rows * kv_vecs, per_act = rows * act_vecs;
  const int kv_segs = 2 * ar.layers;
  const int total = kv_segs * per_kv + per_act + (new_rkeys ? 2 * per_kv : 0);
  for (int base = threadIdx.x; base < total; base += WV_THREADS * WV_BATCH) {
    uint4 val[WV_BATCH];
    uint4* out[WV_BATCH];
#pragma unroll
    for (int k = 0; k < WV_BATCH; ++k) {
      const int idx = base + k * WV_THREADS;
      out[k] = nullptr;
      if (idx >= total) continue;
      const char* seg;                               // arena segment
      const char* fresh;                             // the new row of this child
      int64_t page_bytes, row_bytes;
      int vecs, rem;
      if (idx < kv_segs * per_kv) {
        const int sgi = idx / per_kv;
        rem = idx - sgi * per_kv;
        const int l = sgi < ar.layers ? sgi : sgi - ar.layers;
        seg = (const char*)(sgi < ar.layers ? ar.keys : ar.values) + l * kv_layer;
        fresh = (sgi < ar.layers ? new_keys : new_values) + ((int64_t)l * n + i) * kv_row;
        page_bytes = kv_page, row_bytes = kv_row, vecs = kv_vecs;
      } else if (idx < kv_segs * per_kv + per_act) {
        rem = idx - kv_segs * per_kv;
        seg = (const char*)ar.actions;
        fresh = new_actions + (int64_t)i * act_row;
        page_bytes = act_page, row_bytes = act_row, vecs = act_vecs;
      } else {
        const int r0 = idx - kv_segs * per_kv - per_act;
        const bool second = r0 >= per_kv;
        rem = second ? r0 - per_kv : r0;
        seg = (const char*)(second ? ar.rvalues : ar.rkeys);
        fresh = (second ? new_rvalues : new_rkeys) + (int64_t)i * kv_row;
        page_bytes = kv_page, row_bytes = kv_row, vecs = kv_vecs;
      }
      const int r = rem / vecs, v = rem - r * vecs;
      const char* from = r < offset ? seg + src * page_bytes + r * row_bytes + v * 16
                                    : fresh + v * 16;
      val[k] = __ldg(reinterpret_cast<const uint4*>(from));
      out[k] = reinterpret_cast<uint4*>(const_cast<char*>(seg) + dst * page_bytes +
                                        r * row_bytes + v * 16);
    }
#pragma unroll
    for (int k = 0; k < WV_BATCH; ++k)
      if (out[k]) *out[k] = val[k];
  }
}

// Release pass 1: decrement every page of every handle; remember for each
// page the last scan position (handle-major) that decremented it.
__global__ void cache_release_decrement_kernel(int32_t* __restrict__ refcounts,
                                               int32_t* __restrict__ last_pos, int capacity,
                                               const int32_t* __restrict__ table, int64_t stride,
                                               const int32_t* __restrict__ lengths, int n,
                                               int cols, int page, int32_t* __restrict__ status) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)n * cols) return;
  const int i = (int)(idx / cols), j = (int)(idx % cols);
  if (j >= blocks_for(lengths[i], page)) return;
  const int p = table[(int64_t)i * stride + j];
  if (p < 0 || p >= capacity) { set_status(status, GRS_ERR_BAD_PAGE); return; }
  const int old = atomicSub(&refcounts[p], 1);
  if (old <= 0) set_status(status, GRS_ERR_REFCOUNT);
  atomicMax(&last_pos[p], (int)idx);
}

// Release pass 2 (one CTA): pages whose count reached zero are appended to
// the free list in order of their last decrement; last_pos is then reset.
// Each thread takes REL_PER consecutive scan positions per round, so a round
// is three memory round trips (lengths, table, refcount + last position) and
// one block scan.
constexpr int REL_THREADS = 1024;
constexpr int REL_PER = 8;
__global__ void __launch_bounds__(REL_THREADS) cache_release_collect_kernel(
    const int32_t* __restrict__ refcounts, int32_t* __restrict__ last_pos,
    int32_t* __restrict__ free_list, int32_t* __restrict__ free_count, int capacity,
    const int32_t* __restrict__ table, int64_t stride, const int32_t* __restrict__ lengths,
    int n, int cols, int page) {
  __shared__ int warp_sums[REL_THREADS / 32];
  __shared__ int running;
  if (threadIdx.x == 0) running = *free_count;
  __syncthreads();
  const int64_t total = (int64_t)n * cols;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int held[REL_PER];                   // pages of this thread's last round
  for (int64_t base = 0; base < total; base += (int64_t)REL_THREADS * REL_PER) {
    const int64_t first = base + (int64_t)threadIdx.x * REL_PER;
#pragma unroll
    for (int e = 0; e < REL_PER; ++e) {
      const int64_t idx = first + e;
      held[e] = -1;
      if (idx < total) {
        const int i = (int)(idx / cols), j = (int)(idx % cols);
        if (j < blocks_for(lengths[i], page)) {
          const int cand = table[(int64_t)i * stride + j];
          if (cand >= 0 && cand < capacity) held[e] = cand;
        }
      }
    }
    unsigned flags = 0;
#pragma unroll
    for (int e = 0; e < REL_PER; ++e)
      if (held[e] >= 0 && refcounts[held[e]] == 0 && last_pos[held[e]] == (int)(first + e))
        flags |= 1u << e;
    const int count = __popc(flags);
    int incl = count;                  // block exclusive scan of the counts
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int v = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      warp_sums[lane] = v;             // inclusive over warps
    }
    __syncthreads();
    int pos = running + (warp == 0 ? 0 : warp_sums[warp - 1]) + incl - count;
#pragma unroll
    for (int e = 0; e < REL_PER; ++e)
      if ((flags >> e) & 1u) {
        if (pos < capacity) free_list[pos] = held[e];
        ++pos;
      }
    __syncthreads();
    if (threadIdx.x == 0) running += warp_sums[REL_THREADS / 32 - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) *free_count = min(running, capacity);
  // every flag check has read last_pos (the barrier above): reset it
  if (total <= (int64_t)REL_THREADS * REL_PER) {
#pragma unroll
    for (int e = 0; e < REL_PER; ++e)
      if (held[e] >= 0) last_pos[held[e]] = -1;
  } else {
    for (int64_t idx = threadIdx.x; idx < total; idx += REL_THREADS) {
      const int i = (int)(idx / cols), j = (int)(idx % cols);
      if (j < blocks_for(lengths[i], page)) {
        const int p = table[(int64_t)i * stride + j];
        if (p >= 0 && p < capacity) last_pos[p] = -1;
      }
    }
  }
}

__global__ void cache_init_kernel(int32_t* refcounts, int32_t* free_list, int32_t* free_count,
                                  int32_t* last_pos, int capacity) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < capacity) {
    refcounts[i] = 0;
    free_list[i] = capacity - 1 - i;  // paged_cache.py:75
    last_pos[i] = -1;
  }
  if (i == 0) *free_count = capacity;
}

// Block table validation (paged_cache.py:223-228): each handle's block count
// must equal ceil(length / page).
__global__ void cache_check_lengths_kernel(const int32_t* __restrict__ nblocks,
                                           const int32_t* __restrict__ lengths, int n, int page,
                                           int32_t* __restrict__ status) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n && blocks_for(lengths[i], page) != nblocks[i]) set_status(status, GRS_ERR_LENGTH);
}

// Pop n pages from the top of the free list (request i takes
// free_list[fc - 1 - i], the order the fork kernel uses), give each
// refcount 1 and shrink the free count.  One CTA: the count is read before
// any thread writes it.
__global__ void cache_alloc_kernel(int32_t* __restrict__ refcounts,
                                   const int32_t* __restrict__ free_list,
                                   int32_t* __restrict__ free_count, int capacity, int n,
                                   int32_t* __restrict__ out_pages, int32_t* __restrict__ status) {
  const int fc = *free_count;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int page_id = 0;
    if (i >= fc) {
      set_status(status, GRS_ERR_EXHAUSTED);
    } else {
      const int candidate = free_list[fc - 1 - i];
      if (candidate < 0 || candidate >= capacity || refcounts[candidate] != 0) {
        set_status(status, GRS_ERR_CORRUPT);
      } else {
        page_id = candidate;
        refcounts[page_id] = 1;
      }
    }
    out_pages[i] = page_id;
  }
  __syncthreads();
  if (threadIdx.x == 0) *free_count = fc - min(n, fc);
}

}  // namespace grs

using namespace grs;

extern "C" int grs_cache_alloc(int32_t* refcounts, const int32_t* free_list,
                               int32_t* free_count, int capacity, int n, int32_t* out_pages,
                               int32_t* status, void* stream) {
  if (n <= 0) return GRS_OK;
  if (capacity <= 0) return GRS_ERR_SHAPE;
  cache_alloc_kernel<<<1, 256, 0, grs::counted((cudaStream_t)stream)>>>(
      refcounts, free_list, free_count, capacity, n, out_pages, status);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_cache_init(int32_t* refcounts, int32_t* free_list, int32_t* free_count,
                              int32_t* last_pos, int capacity, void* stream) {
  if (capacity <= 0) return GRS_ERR_SHAPE;
  cache_init_kernel<<<ceil_div(capacity, 256), 256, 0, grs::counted((cudaStream_t)stream)>>>(
      refcounts, free_list, free_count, last_pos, capacity);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_cache_append(int elem_bytes, int32_t* refcounts, int32_t* free_list,
                                int32_t* free_count, int capacity, const int32_t* parent_table,
                                int64_t parent_stride, const int32_t* parent_lengths, int n,
                                int page_size, int32_t* child_table, int64_t child_stride,
                                int32_t* child_lengths, int child_cols, void* keys, void* values,
                                int layers, int heads_x_width, const void* new_keys,
                                const void* new_values, void* actions, int model_width,
                                const void* new_actions, void* readout_keys,
                                void* readout_values, const void* new_readout_keys,
                                const void* new_readout_values, int32_t* status, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (n < 0 || capacity <= 0 || page_size <= 0 || child_cols <= 0 ||
      (elem_bytes != 2 && elem_bytes != 4))
    return GRS_ERR_SHAPE;
  if ((new_readout_keys == nullptr) != (new_readout_values == nullptr)) return GRS_ERR_SHAPE;
  if (n == 0) return GRS_OK;
  cache_fork_kernel<<<ceil_div(n, 128), 128, 0, grs::counted(s)>>>(refcounts, free_list, free_count, capacity,
                                                      parent_table, parent_stride, parent_lengths,
                                                      n, page_size, child_table, child_stride,
                                                      child_lengths, child_cols, status);
  GRS_CUDA_CHECK_LAUNCH();
  CacheArenas ar{keys, values, actions, readout_keys, readout_values, layers, capacity,
                 page_size, heads_x_width, model_width, elem_bytes};
  const bool vec16 =
      ((int64_t)heads_x_width * elem_bytes) % 16 == 0 &&
      ((int64_t)model_width * elem_bytes) % 16 == 0 &&
      ((uintptr_t)keys | (uintptr_t)values | (uintptr_t)actions | (uintptr_t)new_keys |
       (uintptr_t)new_values | (uintptr_t)new_actions | (uintptr_t)readout_keys |
       (uintptr_t)readout_values | (uintptr_t)new_readout_keys |
       (uintptr_t)new_readout_values) % 16 == 0;
  if (vec16)
    cache_write_vec_kernel<<<n, WV_THREADS, 0, grs::counted(s)>>>(
        ar, parent_table, parent_stride, parent_lengths, child_table, child_stride, n,
        (const char*)new_keys, (const char*)new_values, (const char*)new_actions,
        (const char*)new_readout_keys, (const char*)new_readout_values, free_count, status);
  else
    cache_write_kernel<<<n, 128, 0, grs::counted(s)>>>(ar, parent_table, parent_stride, parent_lengths,
                                         child_table, child_stride, n, (const char*)new_keys,
                                         (const char*)new_values, (const char*)new_actions,
                                         (const char*)new_readout_keys,
                                         (const char*)new_readout_values, free_count, status);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_cache_release(int32_t* refcounts, int32_t* free_list, int32_t* free_count,
                                 int32_t* last_pos, int capacity, const int32_t* table,
                                 int64_t stride, const int32_t* lengths, int n, int cols,
                                 int page_size, int32_t* status, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (n < 0 || cols <= 0 || page_size <= 0) return GRS_ERR_SHAPE;
  if (n == 0) return GRS_OK;
  const long long total = (long long)n * cols;
  cache_release_decrement_kernel<<<ceil_div(total, 256), 256, 0, grs::counted(s)>>>(
      refcounts, last_pos, capacity, table, stride, lengths, n, cols, page_size, status);
  GRS_CUDA_CHECK_LAUNCH();
  cache_release_collect_kernel<<<1, REL_THREADS, 0, grs::counted(s)>>>(refcounts, last_pos, free_list,
                                                         free_count, capacity, table, stride,
                                                         lengths, n, cols, page_size);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_cache_check_lengths(const int32_t* nblocks, const int32_t* lengths, int n,
                                       int page_size, int32_t* status, void* stream) {
  if (n <= 0) return GRS_OK;
  cache_check_lengths_kernel<<<ceil_div(n, 256), 256, 0, grs::counted((cudaStream_t)stream)>>>(
      nblocks, lengths, n, page_size, status);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}
