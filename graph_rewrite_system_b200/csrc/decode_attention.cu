// Shared-prefix paged decode attention in one launch of 8-CTA clusters
// (bf16, head width 32, one query per beam and head, an even number of
// heads <= 8, page size a multiple of 16).
//
// Every beam attends to the same `num_shared` s0 node keys/values, to its own
// block-table pages and to an optional current token.  A cluster owns 16
// beams (the M dimension of mma.m16n8k16) and splits their keys into units
// of 16 rows:
//
//   shared units   16 consecutive shared keys
//   page units     16 rows of a page that one or more of the 16 beams hold
//                  in the same block-table column (deduplicated, so a page
//                  the beams share through copy-on-write is read once per
//                  cluster, not once per beam)
//   current unit   the 16 beams' current tokens
//
// Each CTA of the cluster takes every eighth shared unit and every eighth
// page/current unit.  Warp 8 of the CTA is the producer: per unit it issues
// two TMA tile loads (cp.async.bulk.tensor into its own shared memory only),
// one for the K and one for the V rows of all heads, into a ring of five
// stages, completion counted on the stage's "full" mbarrier.  The tensor maps
// view a key row (H*32 bf16) as H/2 chunks of 128 bytes and make the chunk
// the outermost box dimension, so one 8 KB load lands as H/2 tiles of 16 rows
// x 128 bytes with the 128-byte swizzle (conflict-free ldmatrix).  The shared
// units go out at kernel entry; while they land the producer reads the block
// tables, deduplicates the pages per column and publishes this CTA's page
// units (and the beams' lengths) on a "units" mbarrier.  Warps 0-7 are the
// consumers, one per head: they start on the shared units at once, take two
// stages per online-softmax step (masked partial max, sum and P.V for all 16
// beams with ldmatrix-fed mma tiles) and release each stage on its "empty"
// mbarrier.  Each CTA then pushes its partials into the shared memory of the
// beams' owners (CTA beam/2); after one cluster barrier the owners merge the
// eight partials and write the output.
//
// Every mbarrier wait is bounded: a wait that runs out records
// GRS_ERR_TIMEOUT in the caller's status word and the kernel finishes
// without the missing data.  Keys whose page id is outside the cache are
// skipped.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "grs_common.cuh"

namespace cg = cooperative_groups;

namespace grs {

constexpr int DC_CLUSTER = 8;
constexpr int DC_BEAMS = 16;          // beams per cluster (mma M)
constexpr int DC_CONSUMERS = 8;       // warps 0-7, one per head
constexpr int DC_PRODUCER = DC_CONSUMERS;
constexpr int DC_THREADS = (DC_CONSUMERS + 1) * 32;
constexpr int DC_D = 32;
constexpr int DC_UNIT = 16;           // rows per unit / stage (one mma tile of keys)
constexpr int DC_NBUF = 5;            // stages in the ring
constexpr int DC_BOX_BYTES = DC_UNIT * 128;              // one tile: 16 rows x 128 B
constexpr int DC_STAGE_BYTES = 2 * 4 * DC_BOX_BYTES;     // K and V, up to 4 tiles each
constexpr int DC_MAX_COLS = 32;       // block-table columns
constexpr int DC_MAX_UNITS = 64;      // page/current units per CTA
constexpr unsigned long long DC_WAIT_LIMIT_NS = 1000000000ull;   // a wait gives up after 1 s

struct DecodeArgs {
  const __nv_bfloat16* q; int64_t q_sb, q_sh;
  const int32_t* bt; int64_t bt_s; int max_blocks; const int32_t* lengths; int num_pages;
  const uint8_t* cvalid; int has_current;
  int num_shared;
  __nv_bfloat16* out; int64_t o_sb, o_sh;
  int32_t* status;
  int B, H, page; float scale_log2;
};

struct Partial { float m, l, acc[DC_D]; };

__device__ __forceinline__ unsigned smem_addr(const void* p) {
  return (unsigned)__cvta_generic_to_shared(p);
}

// ---- mbarrier and TMA primitives (PTX ISA 8.x) ---------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// bounded wait for the phase with the given parity to complete: gives up
// after DC_WAIT_LIMIT_NS of %globaltimer (try_wait may park the thread per
// poll, so the bound is on elapsed time)
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t start;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(start));
  for (unsigned i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      uint64_t now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (now - start > DC_WAIT_LIMIT_NS) return false;
    }
  }
}
// TMA tile loads into this CTA's own shared memory; the
// innermost coordinate is always 0 (a whole 128-byte chunk)
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int y, int z,
                                            int w, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];\n" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(z), "r"(w),
      "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t r[4], unsigned addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t r[4], unsigned addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^x with the hardware approximation (ex2.approx.ftz: relative error about
// 2^-22, subnormal results flushed to zero); 2^-inf = 0
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Address of the 16-byte chunk `chunk` (0-7) of row `row` in a 16 x 128-byte
// tile written by TMA with 128-byte swizzle (tile base 1024-byte aligned).
__device__ __forceinline__ unsigned swz(unsigned tile, int row, int chunk) {
  return tile + row * 128 + ((chunk ^ (row & 7)) << 4);
}

__global__ void __cluster_dims__(DC_CLUSTER, 1, 1) __launch_bounds__(DC_THREADS, 2)
decode_cluster_kernel(DecodeArgs a, const __grid_constant__ CUtensorMap tm_sk,
                      const __grid_constant__ CUtensorMap tm_sv,
                      const __grid_constant__ CUtensorMap tm_kc,
                      const __grid_constant__ CUtensorMap tm_vc,
                      const __grid_constant__ CUtensorMap tm_ck,
                      const __grid_constant__ CUtensorMap tm_cv) {
  // inbox[slot][head][r]: CTA r's partial for local beam `slot` of this CTA,
  // written by CTA r into this CTA's shared memory
  __shared__ Partial inbox[2][DC_CONSUMERS][DC_CLUSTER];
  __shared__ __align__(8) uint64_t full_bar[DC_NBUF], empty_bar[DC_NBUF], units_bar;
  __shared__ int s_len[DC_BEAMS], s_cur[DC_BEAMS];
  __shared__ int s_bt[DC_MAX_COLS][DC_BEAMS];
  // distinct (column, page) entries: page id, column << 16 | beam mask
  __shared__ int s_entry_page[DC_BEAMS * DC_MAX_COLS];
  __shared__ int s_entry_cm[DC_BEAMS * DC_MAX_COLS];
  __shared__ int s_nunits;
  // this CTA's page/current units: page id (-1: the current unit), first row
  // in the page, beam mask, position of the first row, rows that are keys
  __shared__ int4 s_unit[DC_MAX_UNITS];
  extern __shared__ __align__(1024) unsigned char dyn[];

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int beam0 = (blockIdx.x / DC_CLUSTER) * DC_BEAMS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tig = lane & 3;
  // every CTA of the cluster must be running before another writes into its
  // shared memory: arrive now, wait just before the first remote store
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");

  // the ring, 1024-byte aligned for the 128-byte swizzle
  const unsigned ring = (smem_addr(dyn) + 1023u) & ~1023u;
  const int tiles = (a.H * DC_D + 63) / 64;              // 128-byte tiles per key row
  const unsigned stage_bytes = 2u * tiles * DC_BOX_BYTES;
  const int ns = a.num_shared;
  const int sh_units = (ns + DC_UNIT - 1) / DC_UNIT;
  // this CTA's shared units: rank, rank + 8, ...
  const int my_sh = sh_units > rank ? (sh_units - rank + DC_CLUSTER - 1) / DC_CLUSTER : 0;

  if (tid == 0) {
    for (int i = 0; i < DC_NBUF; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], DC_CONSUMERS);
    }
    mbar_init(&units_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();

  if (warp == DC_PRODUCER) {
    // ---- producer warp: shared stages first, then the block tables, the
    // per-column page dedup and this CTA's page units, then the page stages
    bool ok = true;
    auto produce = [&](int st, int unit_page, int y0) {
      const int buf = st % DC_NBUF;
      if (st >= DC_NBUF)
        ok = __all_sync(0xffffffffu, mbar_wait(&empty_bar[buf], (unsigned)((st / DC_NBUF - 1) & 1)));
      if (ok && lane == 0) {
        mbar_arrive_expect_tx(&full_bar[buf], stage_bytes);
        unsigned char* kdst = dyn + (ring - smem_addr(dyn)) + buf * DC_STAGE_BYTES;
        unsigned char* vdst = kdst + 4 * DC_BOX_BYTES;
        if (unit_page == -2) {              // shared unit: rows y0..y0+15 of [N, chunks, 64]
          tma_load_3d(kdst, &tm_sk, y0, 0, &full_bar[buf]);
          tma_load_3d(vdst, &tm_sv, y0, 0, &full_bar[buf]);
        } else if (unit_page >= 0) {        // page unit: rows y0.. of [pages, page, chunks, 64]
          tma_load_4d(kdst, &tm_kc, y0, 0, unit_page, &full_bar[buf]);
          tma_load_4d(vdst, &tm_vc, y0, 0, unit_page, &full_bar[buf]);
        } else {                            // current unit: the beams' rows of [B, chunks, 64]
          tma_load_3d(kdst, &tm_ck, beam0, 0, &full_bar[buf]);
          tma_load_3d(vdst, &tm_cv, beam0, 0, &full_bar[buf]);
        }
      }
      __syncwarp();
    };
    const int first = min(my_sh, DC_NBUF);          // the ring's first round needs no waits
    for (int i = 0; i < first; ++i) produce(i, -2, (rank + i * DC_CLUSTER) * DC_UNIT);

    // lengths, current-token flags and block-table columns of the 16 beams
    const int cols = a.max_blocks;   // <= DC_MAX_COLS (host-checked)
    if (lane < DC_BEAMS) {
      const int b = beam0 + lane;
      s_len[lane] = b < a.B ? a.lengths[b] : 0;
      s_cur[lane] = (b < a.B && a.has_current) ? (a.cvalid[b] != 0) : 0;
    }
    for (int i = lane; i < cols * DC_BEAMS; i += 32) {
      const int c = i >> 4, j = i & 15, b = beam0 + j;
      s_bt[c][j] = b < a.B ? a.bt[(int64_t)b * a.bt_s + c] : -1;
    }
    __syncwarp();
    // distinct pages per column: lanes 0-15 column c, 16-31 column c+1
    int count = 0;
    for (int c0 = 0; c0 < cols; c0 += 2) {
      const int c = c0 + (lane >> 4), j = lane & 15;
      int p = -1;
      if (c < cols && c * a.page < s_len[j]) {
        p = s_bt[c][j];
        if (p >= a.num_pages) p = -1;
      }
      const unsigned long long key =
          p >= 0 ? (((unsigned long long)(unsigned)p << 1) | (unsigned)(lane >> 4))
                 : ((1ull << 63) | (unsigned)lane);
      const unsigned peers = __match_any_sync(0xffffffffu, key);
      const bool lead = p >= 0 && __ffs(peers) - 1 == lane;
      const unsigned leads = __ballot_sync(0xffffffffu, lead);
      if (lead) {
        const int e = count + __popc(leads & ((1u << lane) - 1u));
        s_entry_page[e] = p;
        s_entry_cm[e] = (c << 16) | ((peers >> (lane & 16)) & 0xFFFF);
      }
      count += __popc(leads);
    }
    __syncwarp();
    // this CTA's page/current units: global unit u = entry * (page/16) +
    // sub-block, the current unit last; CTA r takes u = r, r + 8, ...
    const int per_page = a.page / DC_UNIT;
    const int page_units = count * per_page;
    const int all_units = page_units + (a.has_current ? 1 : 0);
    const int nu = all_units > rank ? (all_units - rank + DC_CLUSTER - 1) / DC_CLUSTER : 0;
    int cur_mask = 0;
    for (int j = 0; j < DC_BEAMS; ++j) cur_mask |= s_cur[j] ? (1 << j) : 0;
    for (int i = lane; i < nu; i += 32) {
      const int u = rank + i * DC_CLUSTER;
      if (u < page_units) {
        const int e = u / per_page, sub = u - e * per_page;
        const int cm = s_entry_cm[e];
        s_unit[i] = make_int4(s_entry_page[e], sub * DC_UNIT, cm & 0xFFFF,
                              (cm >> 16) * a.page + sub * DC_UNIT);
      } else {
        s_unit[i] = make_int4(-1, 0, cur_mask, -1);
      }
    }
    if (lane == 0) s_nunits = nu;
    __syncwarp();
    // publish lengths and units to the consumers (release on arrive)
    if (lane == 0) mbar_arrive(&units_bar);
    for (int i = first; i < my_sh && ok; ++i) produce(i, -2, (rank + i * DC_CLUSTER) * DC_UNIT);
    for (int i = 0; i < nu && ok; ++i) {
      const int4 u = s_unit[i];
      produce(my_sh + i, u.x, u.y);
    }
    if (!ok && lane == 0 && a.status) atomicCAS(a.status, 0, GRS_ERR_TIMEOUT);
    __syncwarp();
  } else {
    // ---- consumers: one warp per head ------------------------------------
    // query fragments of head `warp` for the 16 beams (A operand, rows = beams)
    uint32_t qa[2][4] = {};
    if (warp < a.H) {
      const int r0 = beam0 + g, r1 = beam0 + g + 8;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const int c = ks * 16 + tig * 2;
        const __nv_bfloat16* p0 = a.q + (int64_t)r0 * a.q_sb + (int64_t)warp * a.q_sh + c;
        const __nv_bfloat16* p1 = a.q + (int64_t)r1 * a.q_sb + (int64_t)warp * a.q_sh + c;
        if (r0 < a.B) {
          qa[ks][0] = *reinterpret_cast<const uint32_t*>(p0);
          qa[ks][2] = *reinterpret_cast<const uint32_t*>(p0 + 8);
        }
        if (r1 < a.B) {
          qa[ks][1] = *reinterpret_cast<const uint32_t*>(p1);
          qa[ks][3] = *reinterpret_cast<const uint32_t*>(p1 + 8);
        }
      }
    }
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[4][4] = {};
    const int h = warp;
    bool ok = true;
    int len0 = 0, len1 = 0, nu = 0;

    // consume n (1 or 2) consecutive stages from `st` as one softmax step
    auto consume = [&](int st, int n) {
      int buf[2] = {st % DC_NBUF, (st + 1) % DC_NBUF};
      for (int k = 0; k < n; ++k)
        if (ok) ok = mbar_wait(&full_bar[buf[k]], (unsigned)(((st + k) / DC_NBUF) & 1));
      if (ok && h < a.H) {
        float s[2][2][4] = {};
        const int hc = (h & 1) * 4;                  // chunk of this head in a tile row
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (k >= n) break;
          const unsigned kt = ring + buf[k] * DC_STAGE_BYTES + (h >> 1) * DC_BOX_BYTES;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            uint32_t kf[4];
            ldmatrix_x4(kf, swz(kt, nt * 8 + (lane & 7), hc + (lane >> 3)));
            mma16816(s[k][nt], qa[0], kf[0], kf[1]);
            mma16816(s[k][nt], qa[1], kf[2], kf[3]);
          }
        }
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (k >= n) break;
          const int sk = st + k;
          // visibility of the stage's rows for beams g (v0) and g + 8 (v1)
          int kind, mask = 0xFFFF, pos0 = -1, rows = DC_UNIT;
          if (sk < my_sh) {
            kind = 0;
            rows = min(DC_UNIT, ns - (rank + sk * DC_CLUSTER) * DC_UNIT);
          } else {
            const int4 u = s_unit[sk - my_sh];
            kind = u.x >= 0 ? 1 : 2;
            mask = u.z;
            pos0 = u.w;
          }
          const bool see0 = (mask >> g) & 1, see1 = (mask >> (g + 8)) & 1;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const int r = nt * 8 + tig * 2 + c;
              bool v0, v1;
              if (kind == 0) {
                v0 = v1 = r < rows;
              } else if (kind == 1) {
                v0 = see0 && pos0 + r < len0;
                v1 = see1 && pos0 + r < len1;
              } else {                               // row r is beam r's current token
                v0 = see0 && r == g;
                v1 = see1 && r == g + 8;
              }
              s[k][nt][c] = v0 ? s[k][nt][c] * a.scale_log2 : -INFINITY;
              s[k][nt][2 + c] = v1 ? s[k][nt][2 + c] * a.scale_log2 : -INFINITY;
              mx0 = fmaxf(mx0, s[k][nt][c]);
              mx1 = fmaxf(mx1, s[k][nt][2 + c]);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        // running maxima; a row that has seen no key yet keeps -inf and is
        // exponentiated against 0 instead, so every term is 2^-inf = 0
        const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
        const float e0 = n0 == -INFINITY ? 0.f : n0, e1 = n1 == -INFINITY ? 0.f : n1;
        const float c0 = fast_exp2(m0 - e0), c1 = fast_exp2(m1 - e1);
        float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (k >= n) break;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              s[k][nt][c] = fast_exp2(s[k][nt][c] - e0);
              s[k][nt][2 + c] = fast_exp2(s[k][nt][2 + c] - e1);
              sum0 += s[k][nt][c];
              sum1 += s[k][nt][2 + c];
            }
        }
        // per-lane partial row sums; the quad reduction happens once at the end
        l0 = l0 * c0 + sum0;
        l1 = l1 * c1 + sum1;
        m0 = n0;
        m1 = n1;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          o[nt][0] *= c0; o[nt][1] *= c0; o[nt][2] *= c1; o[nt][3] *= c1;
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (k >= n) break;
          const unsigned vt = ring + buf[k] * DC_STAGE_BYTES + (h >> 1) * DC_BOX_BYTES +
                              4 * DC_BOX_BYTES;
          uint32_t pa[4];
          pa[0] = pack2(s[k][0][0], s[k][0][1]);
          pa[1] = pack2(s[k][0][2], s[k][0][3]);
          pa[2] = pack2(s[k][1][0], s[k][1][1]);
          pa[3] = pack2(s[k][1][2], s[k][1][3]);
#pragma unroll
          for (int dp = 0; dp < 2; ++dp) {
            // four 8x8 tiles: keys 0-7 / 8-15 x dims dp*16 + 0-7 / 8-15
            uint32_t vf[4];
            ldmatrix_x4_trans(vf, swz(vt, (lane & 7) + ((lane >> 3) & 1) * 8,
                                      hc + dp * 2 + (lane >> 4)));
            mma16816(o[2 * dp], pa, vf[0], vf[1]);
            mma16816(o[2 * dp + 1], pa, vf[2], vf[3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0)
        for (int k = 0; k < n; ++k) mbar_arrive(&empty_bar[buf[k]]);
    };

    // the shared stages need no block-table data
    int st = 0;
    for (; st + 1 < my_sh; st += 2) consume(st, 2);
    if (st < my_sh) consume(st++, 1);
    // then the page/current stages, once the producer has published them
    ok = ok && mbar_wait(&units_bar, 0);
    if (ok) {
      nu = s_nunits;
      len0 = s_len[g];
      len1 = s_len[g + 8];
    }
    const int stages = my_sh + nu;
    for (; st + 1 < stages; st += 2) consume(st, 2);
    if (st < stages) consume(st++, 1);
    if (!ok && lane == 0 && a.status) atomicCAS(a.status, 0, GRS_ERR_TIMEOUT);

    // 5. push the partials of beams g and g+8 to their owners
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
    if (h < a.H) {
      Partial* d0 = cluster.map_shared_rank(&inbox[g & 1][h][rank], g >> 1);
      Partial* d1 = cluster.map_shared_rank(&inbox[g & 1][h][rank], (g >> 1) + 4);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int d = nt * 8 + tig * 2;
        *reinterpret_cast<float2*>(&d0->acc[d]) = make_float2(o[nt][0], o[nt][1]);
        *reinterpret_cast<float2*>(&d1->acc[d]) = make_float2(o[nt][2], o[nt][3]);
      }
      if (tig == 0) {
        d0->m = m0; d0->l = l0;
        d1->m = m1; d1->l = l1;
      }
    }
  }
  if (warp == DC_PRODUCER) asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");

  // ---- 6. merge: one cluster barrier makes every pushed partial visible;
  // after it no CTA touches another's shared memory
  cluster.sync();
  if (warp < a.H) {
    const int h = warp, slot = lane >> 4, d = (lane & 15) * 2;
    const int b = beam0 + 2 * rank + slot;
    float mr[DC_CLUSTER], lr[DC_CLUSTER], ar[DC_CLUSTER], br[DC_CLUSTER];
#pragma unroll
    for (int r = 0; r < DC_CLUSTER; ++r) {
      const Partial& p = inbox[slot][h][r];
      mr[r] = p.m;
      lr[r] = p.l;
      const float2 v = *reinterpret_cast<const float2*>(&p.acc[d]);
      ar[r] = v.x;
      br[r] = v.y;
    }
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < DC_CLUSTER; ++r) M = fmaxf(M, mr[r]);
    float L = 0.f, O0 = 0.f, O1 = 0.f;
#pragma unroll
    for (int r = 0; r < DC_CLUSTER; ++r) {
      const float w = fast_exp2(mr[r] - (M == -INFINITY ? 0.f : M));
      L += lr[r] * w;
      O0 += ar[r] * w;
      O1 += br[r] * w;
    }
    if (b < a.B) {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      *reinterpret_cast<__nv_bfloat162*>(a.out + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + d) =
          __floats2bfloat162_rn(O0 * inv, O1 * inv);
    }
  }
}

// ---- grouped decode: one CTA per (32 beams, head), no clusters -------------
//
// The cluster kernel above reads the whole shared prefix once per 16 beams
// and pays for a cross-CTA merge.  Here a CTA owns 32 consecutive beams (two
// mma M tiles of 16) for ONE head and every key those beams see, so the
// shared prefix is read once per 32 beams and per head slice (64 bytes of
// each key row), the pages once per 16-beam tile that holds them, and the
// softmax merge stays inside the CTA.  Beams of a search are stored in
// lineage order, so neighbouring beams share their upper pages.
//
// Staging is plain 16-byte cp.async into shared memory with a 64-byte row
// swizzle (16-byte chunk c of row r at c ^ ((r >> 1) & 3): conflict-free
// ldmatrix over eight consecutive rows).  The shared prefix of the head goes
// out at kernel entry, in chunks of `chunk_rows`; while it lands the CTA reads
// the 32 beams' block tables, two warps deduplicate each M tile's pages per
// column, and the distinct page units (16 rows each; the tile's current tokens
// form one more unit) go out in rounds of `round_units`.  Each thread keeps
// one fixed (K or V, row, 16-byte chunk) position of a unit and walks the
// units, so a copy costs a few instructions.  Warps 0-7 take M tile 0 and
// warps 8-15 M tile 1; the eight warps of a tile take every eighth unit, up
// to four units per online-softmax step (all their scores, one max, one
// rescale; ldmatrix-fed m16n8k16 bf16 mma, fp32 accumulation), and merge
// their eight partials through shared memory at the end.  The kernel has no inter-CTA waits and no spin loops.
constexpr int DG_BEAMS = 32;                  // beams per CTA (two M tiles)
constexpr int DG_WARPS = 16;                  // eight per M tile
constexpr int DG_THREADS = DG_WARPS * 32;
constexpr int DG_MAX_COLS = 32;               // block-table columns
constexpr int DG_TILE_BYTES = DC_UNIT * 64;   // 16 rows x one head of 32 bf16
constexpr int DG_MAX_CHUNK_ROWS = 512;        // shared rows staged at once
constexpr int DG_ROUND_UNITS = 48;            // page/current units staged at once
constexpr int DG_TILE_WARPS = DG_WARPS / 2;
constexpr int DG_STEP = 4;                    // units per online-softmax step
constexpr int DG_MERGE_BYTES = 2 * DG_TILE_WARPS * DC_UNIT * (int)sizeof(Partial);

struct GroupArgs {
  const __nv_bfloat16* q; int64_t q_sb, q_sh;
  const __nv_bfloat16* kc; const __nv_bfloat16* vc; int64_t kc_sp, kc_st, kc_sh;
  const int32_t* bt; int64_t bt_s; int cols; const int32_t* lengths; int num_pages;
  const __nv_bfloat16* ck; const __nv_bfloat16* cv; int64_t ck_sb, ck_sh;
  const uint8_t* cvalid;
  const __nv_bfloat16* sk; const __nv_bfloat16* sv; int num_shared;   // [N, H, 32] contiguous
  __nv_bfloat16* out; int64_t o_sb, o_sh;
  int B, H, page; float scale_log2;
  int chunk_rows;     // shared rows staged at once (a multiple of 16)
  int round_units;    // page/current units staged at once
};

// 16-byte copy into shared memory through L2; a miss brings the surrounding
// 256 bytes into L2 (the other heads' slices of the same key row, which the
// CTAs of those heads read at about the same time)
__device__ __forceinline__ void cp_async16(unsigned dst, const void* src) {
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;\n" ::"r"(dst), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void st_shared_zero16(unsigned dst) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};\n" ::"r"(dst), "r"(0) : "memory");
}
// 16-byte chunk `chunk` (0-3) of row `row` in a tile of 64-byte rows
__device__ __forceinline__ unsigned swz64(unsigned tile, int row, int chunk) {
  return tile + row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4);
}

// one staged unit of 16 key rows as seen by one warp's M tile
struct GroupView {
  unsigned kt, vt;    // K and V tiles in shared memory
  int kind;           // 0 shared, 1 page, 2 current tokens
  int mask;           // beams of the tile that see the unit (page/current)
  int pos0;           // position of the first row (page)
  int rows;           // rows that are keys (shared)
};

__global__ void __launch_bounds__(DG_THREADS, 1) decode_group_kernel(GroupArgs a) {
  __shared__ int s_len[DG_BEAMS], s_cur[DG_BEAMS];
  // element offset of each staged unit's first K/V row for this head (page
  // units), or -1 - m for the current unit of M tile m
  __shared__ int64_t s_uoff[DG_ROUND_UNITS];
  __shared__ int s_bt[DG_MAX_COLS][DG_BEAMS];
  // distinct (column, page) entries per M tile: page id, column << 16 | beam mask
  __shared__ int s_ent_page[2][DC_UNIT * DG_MAX_COLS];
  __shared__ int s_ent_cm[2][DC_UNIT * DG_MAX_COLS];
  __shared__ int s_nent[2], s_curmask[2];
  extern __shared__ __align__(1024) unsigned char dyn[];

  const int h = blockIdx.y;
  const int beam0 = blockIdx.x * DG_BEAMS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int mt = warp / DG_TILE_WARPS, sub = warp % DG_TILE_WARPS;
  const int ns = a.num_shared;
  const unsigned shk = smem_addr(dyn);
  const unsigned shv = shk + a.chunk_rows * 64;
  const unsigned pg = shk + a.chunk_rows * 128;
  Partial* part = reinterpret_cast<Partial*>(dyn + a.chunk_rows * 128 +
                                             a.round_units * 2 * DG_TILE_BYTES);

  // rows r0 .. r0 + chunk_rows - 1 of the shared prefix (head h); rows past
  // the prefix are zero so that masked rows never carry non-finite values.
  // Thread t copies chunk t % 4 of rows t / 4, t / 4 + 128, ... of K and V.
  auto load_shared = [&](int r0) {
    const int rows = min(a.chunk_rows, ns - r0);
    const int rows16 = (rows + DC_UNIT - 1) & ~(DC_UNIT - 1);
    const int c = tid & 3;
    const int64_t row_stride = (int64_t)a.H * DC_D * (DG_THREADS / 4);
    const int64_t off0 = (int64_t)(r0 + (tid >> 2)) * a.H * DC_D + h * DC_D + c * 8;
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const __nv_bfloat16* src = (kv ? a.sv : a.sk) + off0;
      const unsigned tile = kv ? shv : shk;
      for (int r = tid >> 2; r < rows16; r += DG_THREADS / 4, src += row_stride) {
        if (r < rows) cp_async16(swz64(tile, r, c), src);
        else st_shared_zero16(swz64(tile, r, c));
      }
    }
  };

  // 1. the shared prefix goes out first: it needs no block-table data
  if (ns > 0) load_shared(0);
  cp_async_commit();

  // 2. lengths, current-token flags and block-table columns of the 32 beams
  if (tid < DG_BEAMS) {
    const int b = beam0 + tid;
    s_len[tid] = b < a.B ? a.lengths[b] : 0;
    s_cur[tid] = (b < a.B && a.ck) ? (a.cvalid[b] != 0) : 0;
  }
  for (int i = tid; i < a.cols * DG_BEAMS; i += DG_THREADS) {
    const int c = i >> 5, j = i & 31, b = beam0 + j;
    s_bt[c][j] = b < a.B ? a.bt[(int64_t)b * a.bt_s + c] : -1;
  }
  // query fragments (A operand, rows = beams) of this warp's M tile
  uint32_t qa[2][4] = {};
  {
    const int r0 = beam0 + mt * DC_UNIT + g, r1 = r0 + 8;
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      const int c = ks * 16 + tig * 2;
      const __nv_bfloat16* p0 = a.q + (int64_t)r0 * a.q_sb + (int64_t)h * a.q_sh + c;
      const __nv_bfloat16* p1 = a.q + (int64_t)r1 * a.q_sb + (int64_t)h * a.q_sh + c;
      if (r0 < a.B) {
        qa[ks][0] = *reinterpret_cast<const uint32_t*>(p0);
        qa[ks][2] = *reinterpret_cast<const uint32_t*>(p0 + 8);
      }
      if (r1 < a.B) {
        qa[ks][1] = *reinterpret_cast<const uint32_t*>(p1);
        qa[ks][3] = *reinterpret_cast<const uint32_t*>(p1 + 8);
      }
    }
  }
  __syncthreads();

  // 3. distinct pages per column of each M tile (warp m for tile m): lanes
  // 0-15 take column c, lanes 16-31 column c + 1
  if (warp < 2) {
    const int m = warp;
    int count = 0;
    for (int c0 = 0; c0 < a.cols; c0 += 2) {
      const int c = c0 + (lane >> 4), j = m * DC_UNIT + (lane & 15);
      int p = -1;
      if (c < a.cols && c * a.page < s_len[j]) {
        p = s_bt[c][j];
        if (p < 0 || p >= a.num_pages) p = -1;
      }
      const unsigned long long key =
          p >= 0 ? (((unsigned long long)(unsigned)p << 1) | (unsigned)(lane >> 4))
                 : ((1ull << 63) | (unsigned)lane);
      const unsigned peers = __match_any_sync(0xffffffffu, key);
      const bool lead = p >= 0 && __ffs(peers) - 1 == lane;
      const unsigned leads = __ballot_sync(0xffffffffu, lead);
      if (lead) {
        const int e = count + __popc(leads & ((1u << lane) - 1u));
        s_ent_page[m][e] = p;
        s_ent_cm[m][e] = (c << 16) | ((peers >> (lane & 16)) & 0xFFFF);
      }
      count += __popc(leads);
    }
    const unsigned cm = __ballot_sync(0xffffffffu, lane < DC_UNIT && s_cur[m * DC_UNIT + lane]);
    if (lane == 0) {
      s_nent[m] = count;
      s_curmask[m] = (int)cm;
    }
  }
  __syncthreads();

  // units of tile 0 come first, then those of tile 1; per tile: page
  // entry e, 16-row block sb of it, then the current unit (if any beam has one)
  const int per_page = a.page / DC_UNIT;
  const int n0 = s_nent[0] * per_page + (s_curmask[0] ? 1 : 0);
  const int total = n0 + s_nent[1] * per_page + (s_curmask[1] ? 1 : 0);
  // page id (-1: current unit), first row in the page, beam mask, position
  auto unit_info = [&](int u, int& page, int& row0, int& mask, int& pos0, int& m) {
    m = u < n0 ? 0 : 1;
    const int local = u - (m ? n0 : 0);
    if (local < s_nent[m] * per_page) {
      const int e = per_page == 1 ? local : local / per_page, sb = local - e * per_page;
      const int cm = s_ent_cm[m][e];
      page = s_ent_page[m][e];
      row0 = sb * DC_UNIT;
      mask = cm & 0xFFFF;
      pos0 = (cm >> 16) * a.page + row0;
    } else {
      page = -1;
      row0 = 0;
      mask = s_curmask[m];
      pos0 = -1;
    }
  };
  // units u0 .. u0 + nr - 1 into the page slots: first each unit's source
  // offset, then thread t copies (K or V, row, chunk) = position t % 128 of
  // units t / 128, t / 128 + 4, ...
  auto load_round = [&](int u0, int nr) {
    if (tid < nr) {
      int page, row0, mask, pos0, m;
      unit_info(u0 + tid, page, row0, mask, pos0, m);
      s_uoff[tid] = page >= 0
                        ? (int64_t)page * a.kc_sp + (int64_t)row0 * a.kc_st + (int64_t)h * a.kc_sh
                        : (int64_t)(-1 - m);
    }
    __syncthreads();
    const int rem = tid & 127;
    const int kv = rem >> 6, r = (rem >> 2) & 15, c = rem & 3;
    const __nv_bfloat16* cache = kv ? a.vc : a.kc;
    const __nv_bfloat16* cur = kv ? a.cv : a.ck;
    const int64_t page_off = (int64_t)r * a.kc_st + c * 8;
    const unsigned dst0 = swz64(pg + kv * DG_TILE_BYTES, r, c);
    for (int j = tid >> 7; j < nr; j += DG_THREADS / 128) {
      const int64_t off = s_uoff[j];
      const unsigned dst = dst0 + j * 2 * DG_TILE_BYTES;
      if (off >= 0) {
        cp_async16(dst, cache + off + page_off);
      } else {
        const int b = beam0 + (int)(-1 - off) * DC_UNIT + r;
        if (b < a.B) cp_async16(dst, cur + (int64_t)b * a.ck_sb + (int64_t)h * a.ck_sh + c * 8);
        else st_shared_zero16(dst);
      }
    }
  };
  // 4. the first round of page units
  load_round(0, min(total, a.round_units));
  cp_async_commit();

  // ---- online softmax over this warp's units -------------------------------
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[4][4] = {};
  const bool live = beam0 + mt * DC_UNIT < a.B;
  const int len0 = s_len[mt * DC_UNIT + g], len1 = s_len[mt * DC_UNIT + g + 8];

  auto step = [&](int n, const GroupView* v) {
    float s[DG_STEP][2][4] = {};
#pragma unroll
    for (int k = 0; k < DG_STEP; ++k) {
      if (k >= n) break;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        uint32_t kf[4];
        ldmatrix_x4(kf, swz64(v[k].kt, nt * 8 + (lane & 7), lane >> 3));
        mma16816(s[k][nt], qa[0], kf[0], kf[1]);
        mma16816(s[k][nt], qa[1], kf[2], kf[3]);
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int k = 0; k < DG_STEP; ++k) {
      if (k >= n) break;
      // rows of the unit that beams g (vm0) and g + 8 (vm1) see, as 16-bit
      // masks, shifted so that bit nt * 8 + c is this lane's row nt * 8 + tig * 2 + c
      const bool see0 = (v[k].mask >> g) & 1, see1 = (v[k].mask >> (g + 8)) & 1;
      auto first_rows = [](int n) -> unsigned {
        return n >= DC_UNIT ? 0xFFFFu : (n <= 0 ? 0u : (1u << n) - 1u);
      };
      unsigned vm0, vm1;
      if (v[k].kind == 0) {
        vm0 = vm1 = first_rows(v[k].rows);
      } else if (v[k].kind == 1) {
        vm0 = see0 ? first_rows(len0 - v[k].pos0) : 0u;
        vm1 = see1 ? first_rows(len1 - v[k].pos0) : 0u;
      } else {                                     // row r is beam r's current token
        vm0 = see0 ? 1u << g : 0u;
        vm1 = see1 ? 1u << (g + 8) : 0u;
      }
      vm0 >>= tig * 2;
      vm1 >>= tig * 2;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const bool v0 = (vm0 >> (nt * 8 + c)) & 1, v1 = (vm1 >> (nt * 8 + c)) & 1;
          s[k][nt][c] = v0 ? s[k][nt][c] * a.scale_log2 : -INFINITY;
          s[k][nt][2 + c] = v1 ? s[k][nt][2 + c] * a.scale_log2 : -INFINITY;
          mx0 = fmaxf(mx0, s[k][nt][c]);
          mx1 = fmaxf(mx1, s[k][nt][2 + c]);
        }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    // a row that has seen no key yet keeps -inf and is exponentiated against
    // 0 instead, so every term is 2^-inf = 0
    const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
    const float e0 = nm0 == -INFINITY ? 0.f : nm0, e1 = nm1 == -INFINITY ? 0.f : nm1;
    const float c0 = fast_exp2(m0 - e0), c1 = fast_exp2(m1 - e1);
    float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
    for (int k = 0; k < DG_STEP; ++k) {
      if (k >= n) break;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          s[k][nt][c] = fast_exp2(s[k][nt][c] - e0);
          s[k][nt][2 + c] = fast_exp2(s[k][nt][2 + c] - e1);
          sum0 += s[k][nt][c];
          sum1 += s[k][nt][2 + c];
        }
    }
    l0 = l0 * c0 + sum0;
    l1 = l1 * c1 + sum1;
    m0 = nm0;
    m1 = nm1;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      o[nt][0] *= c0; o[nt][1] *= c0; o[nt][2] *= c1; o[nt][3] *= c1;
    }
#pragma unroll
    for (int k = 0; k < DG_STEP; ++k) {
      if (k >= n) break;
      uint32_t pa[4];
      pa[0] = pack2(s[k][0][0], s[k][0][1]);
      pa[1] = pack2(s[k][0][2], s[k][0][3]);
      pa[2] = pack2(s[k][1][0], s[k][1][1]);
      pa[3] = pack2(s[k][1][2], s[k][1][3]);
#pragma unroll
      for (int dp = 0; dp < 2; ++dp) {
        // four 8x8 tiles: keys 0-7 / 8-15 x dims dp*16 + 0-7 / 8-15
        uint32_t vf[4];
        ldmatrix_x4_trans(vf, swz64(v[k].vt, (lane & 7) + ((lane >> 3) & 1) * 8,
                                    dp * 2 + (lane >> 4)));
        mma16816(o[2 * dp], pa, vf[0], vf[1]);
        mma16816(o[2 * dp + 1], pa, vf[2], vf[3]);
      }
    }
  };

  // 5. the shared prefix, chunk by chunk (the first chunk is already in flight)
  for (int r0 = 0; r0 < ns; r0 += a.chunk_rows) {
    if (r0 > 0) {
      __syncthreads();                 // every warp is done with the previous chunk
      load_shared(r0);
      cp_async_commit();
      cp_async_wait<0>();
    } else {
      cp_async_wait<1>();              // the first chunk; the first page round may still land
    }
    __syncthreads();
    const int rows = min(a.chunk_rows, ns - r0);
    const int units = (rows + DC_UNIT - 1) / DC_UNIT;
    if (live)
      for (int u = sub; u < units; u += DG_STEP * DG_TILE_WARPS) {
        GroupView v[DG_STEP];
        int n = 0;
#pragma unroll
        for (int k = 0; k < DG_STEP; ++k) {
          const int uu = u + DG_TILE_WARPS * k;
          if (uu >= units) break;
          v[k] = {shk + uu * DG_TILE_BYTES, shv + uu * DG_TILE_BYTES, 0, 0xFFFF, 0,
                  rows - uu * DC_UNIT};
          n = k + 1;
        }
        step(n, v);
      }
  }

  // 6. the page/current units, round by round (the first round is in flight)
  for (int u0 = 0; u0 < total; u0 += a.round_units) {
    const int nr = min(a.round_units, total - u0);
    if (u0 > 0) {
      __syncthreads();                 // every warp is done with the previous round
      load_round(u0, nr);
      cp_async_commit();
    }
    cp_async_wait<0>();
    __syncthreads();
    // this warp's tile's units inside the round
    const int lo = max(u0, mt == 0 ? 0 : n0), hi = min(u0 + nr, mt == 0 ? n0 : total);
    if (live)
      for (int u = lo + sub; u < hi; u += DG_STEP * DG_TILE_WARPS) {
        GroupView v[DG_STEP];
        int n = 0;
#pragma unroll
        for (int k = 0; k < DG_STEP; ++k) {
          const int uu = u + DG_TILE_WARPS * k;
          if (uu >= hi) break;
          int page, row0, mask, pos0, m;
          unit_info(uu, page, row0, mask, pos0, m);
          const unsigned kt = pg + (uu - u0) * 2 * DG_TILE_BYTES;
          v[k] = {kt, kt + DG_TILE_BYTES, page >= 0 ? 1 : 2, mask, pos0, DC_UNIT};
          n = k + 1;
        }
        step(n, v);
      }
  }
  cp_async_wait<0>();                  // nothing stays in flight past the kernel

  // 7. merge the eight partials of each M tile and write the output
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  {
    Partial* p0 = part + (mt * DG_TILE_WARPS + sub) * DC_UNIT + g;
    Partial* p1 = p0 + 8;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int d = nt * 8 + tig * 2;
      *reinterpret_cast<float2*>(&p0->acc[d]) = make_float2(o[nt][0], o[nt][1]);
      *reinterpret_cast<float2*>(&p1->acc[d]) = make_float2(o[nt][2], o[nt][3]);
    }
    if (tig == 0) {
      p0->m = m0; p0->l = l0;
      p1->m = m1; p1->l = l1;
    }
  }
  __syncthreads();
  {
    const int bb = tid >> 4, d0 = (tid & 15) * 2;   // beam of the CTA, 2 dims
    const int m = bb >> 4, row = bb & 15;
    const Partial* pp = part + m * DG_TILE_WARPS * DC_UNIT + row;
    float M = -INFINITY;
#pragma unroll
    for (int s = 0; s < DG_TILE_WARPS; ++s) M = fmaxf(M, pp[s * DC_UNIT].m);
    const float Me = M == -INFINITY ? 0.f : M;
    float L = 0.f, O0 = 0.f, O1 = 0.f;
#pragma unroll
    for (int s = 0; s < DG_TILE_WARPS; ++s) {
      const Partial& p = pp[s * DC_UNIT];
      const float w = fast_exp2(p.m - Me);
      const float2 acc = *reinterpret_cast<const float2*>(&p.acc[d0]);
      L += p.l * w;
      O0 += acc.x * w;
      O1 += acc.y * w;
    }
    const int b = beam0 + bb;
    if (b < a.B) {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      *reinterpret_cast<__nv_bfloat162*>(a.out + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + d0) =
          __floats2bfloat162_rn(O0 * inv, O1 * inv);
    }
  }
}

// ---- host: tensor maps ----------------------------------------------------
// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// libcuda link), with a small cache keyed by every encoded field.
struct MapKey {
  const void* base; int rank; uint64_t dims[4]; uint64_t strides[3];
  bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// bf16 tensor of `rank` (3 or 4) dims, innermost first: 64-element chunk,
// row, chunk index, [page]; boxes of one chunk x 16 rows x all chunks (x 1)
static bool tile_map(CUtensorMap* out, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes) {
  constexpr int kCache = 32;
  static MapKey keys[kCache];
  static CUtensorMap maps[kCache];
  static int used = 0, next = 0;
  static std::mutex mu;
  MapKey k;
  std::memset(&k, 0, sizeof(k));
  k.base = base;
  k.rank = rank;
  for (int i = 0; i < rank; ++i) k.dims[i] = dims[i];
  for (int i = 0; i < rank - 1; ++i) k.strides[i] = strides_bytes[i];
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (keys[i] == k) {
      *out = maps[i];
      return true;
    }
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t gdim[4], gstr[3];
  cuuint32_t box[4] = {64, DC_UNIT, (cuuint32_t)dims[2], 1}, estr[4] = {1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) gdim[i] = dims[i];
  for (int i = 0; i < rank - 1; ++i) gstr[i] = strides_bytes[i];
  CUtensorMap m;
  if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base), gdim,
         gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  keys[next] = k;
  maps[next] = m;
  next = (next + 1) % kCache;
  used = used < kCache ? used + 1 : kCache;
  *out = m;
  return true;
}

}  // namespace grs

using namespace grs;

// shape and alignment rules shared by both shared-prefix decode kernels
static int check_shared_decode(const void* query, int64_t q_sb, int64_t q_sh,
                               const void* key_cache, const void* value_cache, int64_t kc_sp,
                               int64_t kc_st, int64_t kc_sh, int max_blocks, int num_pages,
                               const void* current_key, const void* current_value,
                               int64_t ck_sb, int64_t ck_sh, const uint8_t* current_valid,
                               const void* shared_key, const void* shared_value, int num_shared,
                               void* output, int64_t o_sb, int64_t o_sh, int heads,
                               int page_size) {
  if (heads <= 0 || heads > DC_CONSUMERS || heads % 2 || page_size <= 0 || page_size % DC_UNIT ||
      num_shared < 0 || num_pages <= 0 || max_blocks <= 0 || max_blocks > DC_MAX_COLS)
    return GRS_ERR_SHAPE;
  // page/current units of one CTA: at most 16 distinct pages per column
  const int64_t max_units =
      (int64_t)DC_BEAMS * max_blocks * (page_size / DC_UNIT) + (current_key ? 1 : 0);
  if ((max_units + DC_CLUSTER - 1) / DC_CLUSTER > DC_MAX_UNITS) return GRS_ERR_SHAPE;
  if ((current_key == nullptr) != (current_value == nullptr) ||
      (current_key == nullptr) != (current_valid == nullptr))
    return GRS_ERR_SHAPE;
  // key rows (all heads of one token) are loaded as tiles: heads adjacent
  // (head stride 32), rows 16-byte aligned
  if (kc_sh != DC_D || (current_key && ck_sh != DC_D)) return GRS_ERR_SHAPE;
  if (((uintptr_t)query | (uintptr_t)key_cache | (uintptr_t)value_cache) & 15) return GRS_ERR_SHAPE;
  if (num_shared > 0 && ((uintptr_t)shared_key | (uintptr_t)shared_value) & 15) return GRS_ERR_SHAPE;
  if ((q_sb | q_sh | kc_sp | kc_st) % 8) return GRS_ERR_SHAPE;
  if (current_key && (((uintptr_t)current_key | (uintptr_t)current_value) & 15 || ck_sb % 8))
    return GRS_ERR_SHAPE;
  if (((uintptr_t)output & 3) || (o_sb | o_sh) % 2) return GRS_ERR_SHAPE;
  return GRS_OK;
}

extern "C" int grs_decode_attention_shared(
    const void* query, int64_t q_sb, int64_t q_sh, const void* key_cache,
    const void* value_cache, int64_t kc_sp, int64_t kc_st, int64_t kc_sh,
    const int32_t* block_table, int64_t bt_stride, int max_blocks, const int32_t* lengths,
    int num_pages, const void* current_key, const void* current_value, int64_t ck_sb,
    int64_t ck_sh, const uint8_t* current_valid, const void* shared_key,
    const void* shared_value, int num_shared, void* output, int64_t o_sb, int64_t o_sh,
    int batch, int heads, int page_size, int32_t* status, void* stream) {
  if (batch <= 0) return GRS_OK;
  if (int rc = check_shared_decode(query, q_sb, q_sh, key_cache, value_cache, kc_sp, kc_st,
                                   kc_sh, max_blocks, num_pages, current_key, current_value,
                                   ck_sb, ck_sh, current_valid, shared_key, shared_value,
                                   num_shared, output, o_sb, o_sh, heads, page_size))
    return rc;
  GroupArgs a{(const __nv_bfloat16*)query, q_sb, q_sh, (const __nv_bfloat16*)key_cache,
              (const __nv_bfloat16*)value_cache, kc_sp, kc_st, kc_sh, block_table, bt_stride,
              max_blocks, lengths, num_pages, (const __nv_bfloat16*)current_key,
              (const __nv_bfloat16*)current_value, ck_sb, ck_sh, current_valid,
              (const __nv_bfloat16*)shared_key, (const __nv_bfloat16*)shared_value, num_shared,
              (__nv_bfloat16*)output, o_sb, o_sh, batch, heads, page_size,
              1.4426950408889634f / sqrtf(32.f), 0, DG_ROUND_UNITS};
  a.chunk_rows = num_shared > 0
                     ? min(DG_MAX_CHUNK_ROWS, (num_shared + DC_UNIT - 1) / DC_UNIT * DC_UNIT)
                     : 0;
  const size_t smem = (size_t)a.chunk_rows * 128 + (size_t)a.round_units * 2 * DG_TILE_BYTES +
                      DG_MERGE_BYTES;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(decode_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         DG_MAX_CHUNK_ROWS * 128 + DG_ROUND_UNITS * 2 * DG_TILE_BYTES +
                             DG_MERGE_BYTES);
    attr[dev] = true;
  }
  const dim3 grid((batch + DG_BEAMS - 1) / DG_BEAMS, heads);
  decode_group_kernel<<<grid, DG_THREADS, smem, grs::counted((cudaStream_t)stream)>>>(a);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_decode_attention_shared_cluster(
    const void* query, int64_t q_sb, int64_t q_sh, const void* key_cache,
    const void* value_cache, int64_t kc_sp, int64_t kc_st, int64_t kc_sh,
    const int32_t* block_table, int64_t bt_stride, int max_blocks, const int32_t* lengths,
    int num_pages, const void* current_key, const void* current_value, int64_t ck_sb,
    int64_t ck_sh, const uint8_t* current_valid, const void* shared_key,
    const void* shared_value, int num_shared, void* output, int64_t o_sb, int64_t o_sh,
    int batch, int heads, int page_size, int32_t* status, void* stream) {
  if (batch <= 0) return GRS_OK;
  if (int rc = check_shared_decode(query, q_sb, q_sh, key_cache, value_cache, kc_sp, kc_st,
                                   kc_sh, max_blocks, num_pages, current_key, current_value,
                                   ck_sb, ck_sh, current_valid, shared_key, shared_value,
                                   num_shared, output, o_sb, o_sh, heads, page_size))
    return rc;
  // a key row of H*32 elements as H/2 chunks of 64 (128 bytes)
  const uint64_t chunks = (uint64_t)heads / 2;
  CUtensorMap tm_kc, tm_vc, tm_sk, tm_sv, tm_ck, tm_cv;
  {
    const uint64_t dims[4] = {64, (uint64_t)page_size, chunks, (uint64_t)num_pages};
    const uint64_t str[3] = {(uint64_t)kc_st * 2, 128, (uint64_t)kc_sp * 2};
    if (!tile_map(&tm_kc, key_cache, 4, dims, str) || !tile_map(&tm_vc, value_cache, 4, dims, str))
      return GRS_ERR_SHAPE;
  }
  tm_sk = tm_sv = tm_ck = tm_cv = tm_kc;                 // placeholders for absent inputs
  if (num_shared > 0) {
    const uint64_t dims[3] = {64, (uint64_t)num_shared, chunks};
    const uint64_t str[2] = {(uint64_t)heads * DC_D * 2, 128};
    if (!tile_map(&tm_sk, shared_key, 3, dims, str) || !tile_map(&tm_sv, shared_value, 3, dims, str))
      return GRS_ERR_SHAPE;
  }
  if (current_key) {
    const uint64_t dims[3] = {64, (uint64_t)batch, chunks};
    const uint64_t str[2] = {(uint64_t)ck_sb * 2, 128};
    if (!tile_map(&tm_ck, current_key, 3, dims, str) || !tile_map(&tm_cv, current_value, 3, dims, str))
      return GRS_ERR_SHAPE;
  }
  DecodeArgs a{(const __nv_bfloat16*)query, q_sb, q_sh, block_table, bt_stride, max_blocks,
               lengths, num_pages, current_valid, current_key != nullptr, num_shared,
               (__nv_bfloat16*)output, o_sb, o_sh, status, batch, heads, page_size,
               1.4426950408889634f / sqrtf(32.f)};
  const int clusters = (batch + DC_BEAMS - 1) / DC_BEAMS;
  // the ring plus up to 1 KB to align it to 1024 bytes
  const size_t smem = (size_t)DC_NBUF * DC_STAGE_BYTES + 1024;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(decode_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    attr[dev] = true;
  }
  decode_cluster_kernel<<<clusters * DC_CLUSTER, DC_THREADS, smem, grs::counted((cudaStream_t)stream)>>>(
      a, tm_sk, tm_sv, tm_kc, tm_vc, tm_ck, tm_cv);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}
