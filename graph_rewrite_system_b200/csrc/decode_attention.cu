// Shared-prefix paged decode attention in one launch of 8-CTA clusters
// (bf16, head width 32, one query per beam and head).
//
// Every beam attends to the same `num_shared` s0 node keys/values and to its
// own block-table pages (+ an optional current token).  A cluster owns 16
// beams.  Phase 1: CTA r of the cluster computes, for all 16 beams and every
// head, the softmax partial (max, sum, P.V) over its 1/8 slice of the shared
// keys with mma.m16n8k16 tiles (the 16 beams are the M dimension), so the
// shared prefix is read from L2 once per CTA instead of once per beam.
// The slice is staged into shared memory with cp.async first, and phase 2
// runs while it lands: CTA r computes the partial over the pages of its two
// beams, one warp per (beam, head), a quad of lanes per key, 16-byte loads,
// eight keys in flight per lane.  Each CTA pushes the phase-1 partials of
// every beam into the shared memory of the beam's owner (CTA beam/2); phase
// 3, after one cluster barrier, merges the eight pushed partials with the
// owner's page partial from local shared memory and writes the output.  Keys
// whose page id is outside the cache are skipped.
#include <cooperative_groups.h>

#include "grs_common.cuh"

namespace cg = cooperative_groups;

namespace grs {

constexpr int DC_CLUSTER = 8;
constexpr int DC_BEAMS = 16;          // beams per cluster (mma M)
constexpr int DC_WARPS = 8;
constexpr int DC_D = 32;
constexpr int DC_MAXH = DC_WARPS;  // heads <= warps
constexpr int DC_MAX_CHUNK = 64;      // shared keys per CTA

struct DecodeArgs {
  const __nv_bfloat16* q; int64_t q_sb, q_sh;
  const __nv_bfloat16* kc; const __nv_bfloat16* vc; int64_t kc_sp, kc_st, kc_sh;
  const int32_t* bt; int64_t bt_s; int max_blocks; const int32_t* lengths; int num_pages;
  const __nv_bfloat16* ck; const __nv_bfloat16* cv; int64_t ck_sb, ck_sh; const uint8_t* cvalid;
  const __nv_bfloat16* sk; const __nv_bfloat16* sv; int num_shared; int chunk;
  __nv_bfloat16* out; int64_t o_sb, o_sh;
  int B, H, page; float scale_log2;
};

struct Partial { float m, l, acc[DC_D]; };

// Shared-key slice staged in shared memory: [key][head][32] rows padded to
// H*32+8 elements so the eight fragment rows of an mma tile hit distinct banks.
__device__ __forceinline__ int stage_stride(int H) { return H * DC_D + 8; }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  const unsigned saddr = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(gmem),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], const uint32_t b[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t pack2raw(__nv_bfloat16 lo, __nv_bfloat16 hi) {
  __nv_bfloat162 v; v.x = lo; v.y = hi;
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void unpack8(const uint4 x, float out[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    out[2 * j] = f.x;
    out[2 * j + 1] = f.y;
  }
}

__device__ __forceinline__ float dot8(const uint4 x, const float q[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x);
  float d = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    d += q[2 * j] * f.x + q[2 * j + 1] * f.y;
  }
  return d;
}

__device__ __forceinline__ void axpy8(const uint4 x, float p, float acc[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    acc[2 * j] += p * f.x;
    acc[2 * j + 1] += p * f.y;
  }
}

__global__ void __cluster_dims__(DC_CLUSTER, 1, 1) __launch_bounds__(DC_WARPS * 32, 2)
decode_cluster_kernel(DecodeArgs a) {
  // inbox[slot][head][r]: CTA r's shared-key partial for local beam slot
  // `slot` of this CTA, written by CTA r into this CTA's shared memory
  __shared__ Partial inbox[2][DC_MAXH][DC_CLUSTER];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int cluster_id = blockIdx.x / DC_CLUSTER;
  const int beam0 = cluster_id * DC_BEAMS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  // every CTA of the cluster must be running before another writes into its
  // shared memory: arrive now, wait just before the first remote store
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");

  // ---- stage this CTA's shared-key slice (asynchronous, zero-filled) --------
  extern __shared__ __align__(16) unsigned char dyn[];
  __nv_bfloat16* ks_s = reinterpret_cast<__nv_bfloat16*>(dyn);
  const int sstride = stage_stride(a.H);
  __nv_bfloat16* vs_s = ks_s + (size_t)a.chunk * sstride;
  const int k0 = rank * a.chunk;
  const int kn = max(0, min(a.chunk, a.num_shared - k0));
  {
    const int vec_per_key = a.H * DC_D / 8;              // 16-byte vectors per key row
    const int total = a.chunk * vec_per_key;
    for (int i = threadIdx.x; i < total; i += DC_WARPS * 32) {
      const int key = i / vec_per_key, v = i % vec_per_key;
      const int h = v / (DC_D / 8), part = v % (DC_D / 8);
      const bool ok = key < kn;
      const int64_t goff = ((int64_t)(k0 + (ok ? key : 0)) * a.H + h) * DC_D + part * 8;
      const size_t soff = (size_t)key * sstride + h * DC_D + part * 8;
      cp_async16(ks_s + soff, a.sk + (ok ? goff : 0), ok ? 16 : 0);
      cp_async16(vs_s + soff, a.sv + (ok ? goff : 0), ok ? 16 : 0);
    }
  }

  // ---- phase 2: the pages of this CTA's two beams ---------------------------
  // warp task t = warp + 8*slot: local beam 2*rank + t / H, head t % H.  A key
  // row (64 bytes of one head) is split over a quad of lanes, 16 bytes each;
  // quad g takes keys g, g+8, ..., g+56 of a 64-key block, so every lane has
  // eight K loads (to registers) and eight V copies (cp.async to a per-warp
  // shared buffer) in flight before it uses one.  The lengths,
  // validity flags and the first block's page ids of both slots are
  // loaded up front (page ids speculatively, clamped to the table width), so
  // each slot costs one dependent round trip to memory: its query and
  // current token are loaded with its keys, and the current token is folded
  // in after the pages.  Lane (g, t) ends holding dimension t*8 + g of the
  // partial, which goes to shared memory for phase 3.
  const int tasks = 2 * a.H;
  __nv_bfloat16* vbuf = vs_s + (size_t)a.chunk * sstride + warp * 64 * DC_D;
  // per warp and slot: history length, current-token flag, the first
  // block's page ids (at most 64) and, after the pages, the partial
  __shared__ int first_pages[DC_WARPS][2][64];
  __shared__ int slot_len[DC_WARPS][2], slot_cur[DC_WARPS][2];
  __shared__ Partial page_part[DC_WARPS][2];
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    const int t = warp + slot * DC_WARPS;
    const int b = t < tasks ? beam0 + 2 * rank + t / a.H : a.B;
    const bool live = b < a.B;
    const int past = live ? __ldg(a.lengths + b) : 0;
    const int cur = live && a.ck != nullptr && __ldg(a.cvalid + b) != 0;
    if (lane == 0) {
      slot_len[warp][slot] = past;
      slot_cur[warp][slot] = cur;
    }
    const int first_blocks = min((64 + a.page - 1) / a.page, a.max_blocks);
#pragma unroll
    for (int j = lane; j < 64; j += 32)
      if (live && j < first_blocks)
        first_pages[warp][slot][j] = __ldg(a.bt + (int64_t)b * a.bt_s + j);
  }
  __syncwarp();
#pragma unroll 1
  for (int slot = 0; slot < 2; ++slot) {
    const int t = warp + slot * DC_WARPS;
    const int b = t < tasks ? beam0 + 2 * rank + t / a.H : a.B, h = t % a.H;
    float m = -INFINITY, l = 0.f, acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    // the query is not needed to address the keys: load it with them
    const uint4 qpk = b < a.B ? __ldg(reinterpret_cast<const uint4*>(
                                    a.q + (int64_t)b * a.q_sb + (int64_t)h * a.q_sh + tig * 8))
                              : make_uint4(0, 0, 0, 0);
    const int past = slot_len[warp][slot];
    const bool cur = slot_cur[warp][slot] != 0;
    uint4 ckr = make_uint4(0, 0, 0, 0), cvr = ckr;
    if (cur) {
      const int64_t off = (int64_t)b * a.ck_sb + (int64_t)h * a.ck_sh + tig * 8;
      ckr = __ldg(reinterpret_cast<const uint4*>(a.ck + off));
      cvr = __ldg(reinterpret_cast<const uint4*>(a.cv + off));
    }
    for (int base = 0; base < past; base += 64) {
      // K rows to registers; V rows to this warp's shared buffer (each lane
      // reads back only the 16-byte pieces it copied itself)
      uint4 kr[8];
      bool ok[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int tk = base + g + 8 * u;
        ok[u] = false;
        kr[u] = make_uint4(0, 0, 0, 0);
        if (tk < past) {
          const int pg = base == 0 ? first_pages[warp][slot][tk / a.page]
                                   : __ldg(a.bt + (int64_t)b * a.bt_s + tk / a.page);
          if (pg >= 0 && pg < a.num_pages) {
            const int64_t off = (int64_t)pg * a.kc_sp + (int64_t)(tk % a.page) * a.kc_st +
                                (int64_t)h * a.kc_sh + tig * 8;
            kr[u] = __ldg(reinterpret_cast<const uint4*>(a.kc + off));
            cp_async16(vbuf + (u * 8 + g) * DC_D + tig * 8, a.vc + off, 16);
            ok[u] = true;
          }
        }
      }
      float qv[8];
      unpack8(qpk, qv);
      float sc[8];
      float cm = -INFINITY;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        float d = dot8(kr[u], qv);
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        sc[u] = ok[u] ? d * a.scale_log2 : -INFINITY;
        cm = fmaxf(cm, sc[u]);
      }
      cm = warp_max(cm);
      const float nm = fmaxf(m, cm);
      const float corr = (m == -INFINITY || nm == -INFINITY) ? 0.f : exp2f(m - nm);
      l *= corr;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] *= corr;
      cp_async_wait_all();
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (ok[u]) {
          const float p = exp2f(sc[u] - nm);
          l += p;
          axpy8(*reinterpret_cast<const uint4*>(vbuf + (u * 8 + g) * DC_D + tig * 8), p, acc);
        }
      }
      m = nm;
    }
    // the current token: every quad scores it, quad 0 alone accumulates it
    float qv[8];
    unpack8(qpk, qv);
    float d = dot8(ckr, qv);
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    d += __shfl_xor_sync(0xffffffffu, d, 2);
    if (cur) {
      const float sc = d * a.scale_log2;
      const float nm = fmaxf(m, sc);
      const float corr = m == -INFINITY ? 0.f : exp2f(m - nm);
      const float p = g == 0 ? exp2f(sc - nm) : 0.f;
      l = l * corr + p;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] *= corr;
      axpy8(cvr, p, acc);
      m = nm;
    }
    // sum over the eight quads; the halving exchange leaves lane (g, t)
    // with element g of its quad slice, i.e. dimension t*8 + g
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
#pragma unroll
    for (int half = 16, n = 4; half >= 4; half >>= 1, n >>= 1) {
      const bool upper = (lane & half) != 0;
#pragma unroll
      for (int e = 0; e < n; ++e) {
        const float send = upper ? acc[e] : acc[e + n];
        const float keep = upper ? acc[e + n] : acc[e];
        acc[e] = keep + __shfl_xor_sync(0xffffffffu, send, half);
      }
    }
    page_part[warp][slot].acc[tig * 8 + g] = acc[0];
    if (lane == 0) {
      page_part[warp][slot].m = m;
      page_part[warp][slot].l = l;
    }
  }

  // ---- phase 1: shared-key slice, all 16 beams, mma tiles from shared memory
  cp_async_wait_all();
  __syncthreads();
  asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
  for (int h = warp; h < a.H; h += DC_WARPS) {
    uint32_t qa[2][4];
    const int r0 = beam0 + g, r1 = beam0 + g + 8;
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      const int c = ks * 16 + tig * 2;
      const __nv_bfloat16* p0 = a.q + (int64_t)r0 * a.q_sb + (int64_t)h * a.q_sh + c;
      const __nv_bfloat16* p1 = a.q + (int64_t)r1 * a.q_sb + (int64_t)h * a.q_sh + c;
      qa[ks][0] = r0 < a.B ? *reinterpret_cast<const uint32_t*>(p0) : 0u;
      qa[ks][1] = r1 < a.B ? *reinterpret_cast<const uint32_t*>(p1) : 0u;
      qa[ks][2] = r0 < a.B ? *reinterpret_cast<const uint32_t*>(p0 + 8) : 0u;
      qa[ks][3] = r1 < a.B ? *reinterpret_cast<const uint32_t*>(p1 + 8) : 0u;
    }
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[4][4] = {};
    for (int base = 0; base < kn; base += 16) {
      float s[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
        const __nv_bfloat16* kr = ks_s + (size_t)(base + nt * 8 + g) * sstride + h * DC_D;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          uint32_t bf[2];
          bf[0] = *reinterpret_cast<const uint32_t*>(kr + ks * 16 + tig * 2);
          bf[1] = *reinterpret_cast<const uint32_t*>(kr + ks * 16 + tig * 2 + 8);
          mma16816(s[nt], qa[ks], bf);
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const bool ok = base + nt * 8 + tig * 2 + c < kn;
          s[nt][c] = ok ? s[nt][c] * a.scale_log2 : -INFINITY;
          s[nt][2 + c] = ok ? s[nt][2 + c] * a.scale_log2 : -INFINITY;
          mx0 = fmaxf(mx0, s[nt][c]);
          mx1 = fmaxf(mx1, s[nt][2 + c]);
        }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
      const float c0 = m0 == -INFINITY ? 0.f : exp2f(m0 - n0);
      const float c1 = m1 == -INFINITY ? 0.f : exp2f(m1 - n1);
      float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          s[nt][c] = s[nt][c] == -INFINITY ? 0.f : exp2f(s[nt][c] - n0);
          s[nt][2 + c] = s[nt][2 + c] == -INFINITY ? 0.f : exp2f(s[nt][2 + c] - n1);
          sum0 += s[nt][c];
          sum1 += s[nt][2 + c];
        }
      sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
      sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
      sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
      sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
      l0 = l0 * c0 + sum0;
      l1 = l1 * c1 + sum1;
      m0 = n0;
      m1 = n1;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        o[nt][0] *= c0; o[nt][1] *= c0; o[nt][2] *= c1; o[nt][3] *= c1;
      }
      uint32_t pa[4];
      pa[0] = pack2(s[0][0], s[0][1]);
      pa[1] = pack2(s[0][2], s[0][3]);
      pa[2] = pack2(s[1][0], s[1][1]);
      pa[3] = pack2(s[1][2], s[1][3]);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int dim = h * DC_D + nt * 8 + g;
        const int kr0 = base + tig * 2, kr1 = base + tig * 2 + 8;
        uint32_t bf[2];
        bf[0] = pack2raw(vs_s[(size_t)kr0 * sstride + dim], vs_s[(size_t)(kr0 + 1) * sstride + dim]);
        bf[1] = pack2raw(vs_s[(size_t)kr1 * sstride + dim], vs_s[(size_t)(kr1 + 1) * sstride + dim]);
        mma16816(o[nt], pa, bf);
      }
    }
    // push the partials of beams g and g+8 to their owners (CTA beam/2)
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

  // ---- phase 3: merge with the eight prefix partials ------------------------
  // One cluster barrier makes every pushed partial visible; after it no CTA
  // touches another's shared memory, so none has to wait for the others.
  cluster.sync();
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    const int t = warp + slot * DC_WARPS;
    if (t >= tasks) continue;
    const int ls = t / a.H, h = t % a.H;
    const int b = beam0 + 2 * rank + ls;
    // lane (g, t) holds dimension t*8 + g of the page partial
    const int dim = tig * 8 + g;
    float mr[DC_CLUSTER], lr[DC_CLUSTER], ar[DC_CLUSTER];
#pragma unroll
    for (int r = 0; r < DC_CLUSTER; ++r) {
      const Partial& p = inbox[ls][h][r];
      mr[r] = p.m;
      lr[r] = p.l;
      ar[r] = p.acc[dim];
    }
    const Partial& pp = page_part[warp][slot];
    const float m = pp.m;
    float M = m;
#pragma unroll
    for (int r = 0; r < DC_CLUSTER; ++r) M = fmaxf(M, mr[r]);
    const float wp = m == -INFINITY ? 0.f : exp2f(m - M);
    float L = pp.l * wp, O = pp.acc[dim] * wp;
#pragma unroll
    for (int r = 0; r < DC_CLUSTER; ++r) {
      const float w = mr[r] == -INFINITY ? 0.f : exp2f(mr[r] - M);
      L += lr[r] * w;
      O += ar[r] * w;
    }
    if (b < a.B)
      a.out[(int64_t)b * a.o_sb + (int64_t)h * a.o_sh + dim] =
          __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
  }
}

}  // namespace grs

using namespace grs;

extern "C" int grs_decode_attention_shared(
    const void* query, int64_t q_sb, int64_t q_sh, const void* key_cache,
    const void* value_cache, int64_t kc_sp, int64_t kc_st, int64_t kc_sh,
    const int32_t* block_table, int64_t bt_stride, int max_blocks, const int32_t* lengths,
    int num_pages,
    const void* current_key, const void* current_value, int64_t ck_sb, int64_t ck_sh,
    const uint8_t* current_valid, const void* shared_key, const void* shared_value,
    int num_shared, void* output, int64_t o_sb, int64_t o_sh, int batch, int heads,
    int page_size, void* stream) {
  if (batch <= 0) return GRS_OK;
  // two (beam, head) page tasks per warp: heads <= DC_WARPS
  if (heads <= 0 || heads > DC_WARPS || page_size <= 0 || num_shared < 0 || max_blocks <= 0)
    return GRS_ERR_SHAPE;
  int chunk = (num_shared + DC_CLUSTER - 1) / DC_CLUSTER;
  chunk = (chunk + 15) / 16 * 16;
  if (chunk > DC_MAX_CHUNK) return GRS_ERR_SHAPE;
  if ((current_key == nullptr) != (current_value == nullptr) ||
      (current_key == nullptr) != (current_valid == nullptr))
    return GRS_ERR_SHAPE;
  if (((uintptr_t)query | (uintptr_t)key_cache | (uintptr_t)value_cache) & 15) return GRS_ERR_SHAPE;
  if (num_shared > 0 && ((uintptr_t)shared_key | (uintptr_t)shared_value) & 15) return GRS_ERR_SHAPE;
  if ((q_sb | q_sh | kc_sp | kc_st | kc_sh) % 8) return GRS_ERR_SHAPE;
  if (current_key && (((uintptr_t)current_key | (uintptr_t)current_value) & 15 || (ck_sb | ck_sh) % 8))
    return GRS_ERR_SHAPE;
  DecodeArgs a{(const __nv_bfloat16*)query, q_sb, q_sh, (const __nv_bfloat16*)key_cache,
               (const __nv_bfloat16*)value_cache, kc_sp, kc_st, kc_sh, block_table, bt_stride,
               max_blocks, lengths, num_pages, (const __nv_bfloat16*)current_key,
               (const __nv_bfloat16*)current_value, ck_sb, ck_sh, current_valid,
               (const __nv_bfloat16*)shared_key, (const __nv_bfloat16*)shared_value, num_shared,
               chunk, (__nv_bfloat16*)output, o_sb, o_sh, batch, heads, page_size,
               1.4426950408889634f / sqrtf(32.f)};
  const int clusters = (batch + DC_BEAMS - 1) / DC_BEAMS;
  // staged shared-key slice (K and V) + one 64-key V buffer per warp
  const size_t smem = ((size_t)2 * chunk * (heads * DC_D + 8) + DC_WARPS * 64 * DC_D) *
                      sizeof(__nv_bfloat16);
  if (smem > 96 * 1024) return GRS_ERR_SHAPE;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(decode_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         96 * 1024);
    attr[dev] = true;
  }
  decode_cluster_kernel<<<clusters * DC_CLUSTER, DC_WARPS * 32, smem, (cudaStream_t)stream>>>(a);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}
