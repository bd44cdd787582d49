// Paged attention over block-table K/V pages (reference paged_attention.py).
//
// Two kernels:
//  * rows kernel: one warp per (beam, head, query) row, online softmax over
//    32-key chunks, lane-per-key scores and lane-per-dim P.V.  Any head width
//    up to 128, bf16 or fp32 arenas, optional current token (causal decode,
//    paged_attention.py:101-132) and an optional shared key/value prefix that
//    every beam attends to before its own pages.
//  * readout kernel (bf16, head width 32): one CTA per beam stages 64-token
//    K/V tiles of all heads in shared memory once and runs the node queries
//    through mma.m16n8k16 tiles with an online softmax, so K/V is read from
//    HBM once per beam instead of once per query.
#include "grs_common.cuh"

namespace grs {

template <typename T, int D>
struct RowsArgs {
  const T* q; int64_t q_sb, q_sh, q_sq;
  const T* kc; const T* vc; int64_t kc_sp, kc_st, kc_sh;
  const int32_t* bt; int64_t bt_s; const int32_t* lengths; int num_pages;
  const T* ck; const T* cv; int64_t ck_sb, ck_sh; const uint8_t* cvalid;
  const T* sk; const T* sv; int num_shared;
  T* out; int64_t o_sb, o_sh, o_sq;
  int B, H, Q, page; float scale_log2;
};

template <int D>
struct LaneDims { static constexpr int N = (D + 31) / 32; };

template <typename T, int D>
__device__ __forceinline__ const T* token_key(const RowsArgs<T, D>& a, int b, int h, int t,
                                              int past, bool is_v) {
  // token order: shared prefix, paged history [0, past), current token.
  if (t < a.num_shared) {
    const T* base = is_v ? a.sv : a.sk;
    return base + ((int64_t)t * a.H + h) * D;
  }
  t -= a.num_shared;
  if (t < past) {
    int page = a.bt[(int64_t)b * a.bt_s + t / a.page];
    if (page < 0 || page >= a.num_pages) return nullptr;  // not a cache page: no key
    const T* base = is_v ? a.vc : a.kc;
    return base + (int64_t)page * a.kc_sp + (int64_t)(t % a.page) * a.kc_st + (int64_t)h * a.kc_sh;
  }
  const T* base = is_v ? a.cv : a.ck;
  return base + (int64_t)b * a.ck_sb + (int64_t)h * a.ck_sh;
}

template <typename T, int D>
__global__ void __launch_bounds__(256) paged_attention_rows_kernel(RowsArgs<T, D> a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t total = (int64_t)a.B * a.H * a.Q;
  if (row >= total) return;
  const int qi = (int)(row % a.Q);
  const int h = (int)((row / a.Q) % a.H);
  const int b = (int)(row / ((int64_t)a.Q * a.H));

  float qv[D];
  const T* qp = a.q + (int64_t)b * a.q_sb + (int64_t)h * a.q_sh + (int64_t)qi * a.q_sq;
#pragma unroll
  for (int d = 0; d < D; ++d) qv[d] = to_float(qp[d]);

  const int past = a.lengths[b];
  const bool cur = a.ck != nullptr && a.cvalid[b] != 0;
  const int T_total = a.num_shared + past + (cur ? 1 : 0);

  constexpr int ND = LaneDims<D>::N;
  float acc[ND];
#pragma unroll
  for (int i = 0; i < ND; ++i) acc[i] = 0.f;
  float m = -INFINITY, l = 0.f;

  for (int base = 0; base < T_total; base += 32) {
    const int t = base + lane;
    float s = -INFINITY;
    const T* kp = t < T_total ? token_key(a, b, h, t, past, false) : nullptr;
    if (kp) {
      float dot = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) dot += qv[d] * to_float(kp[d]);
      s = dot * a.scale_log2;
    }
    const float cmax = warp_max(s);
    const float m_new = fmaxf(m, cmax);
    const float p = kp ? exp2f(s - m_new) : 0.f;
    const float corr = (m == -INFINITY || m_new == -INFINITY) ? 0.f : exp2f(m - m_new);
    l = l * corr + warp_sum(p);
#pragma unroll
    for (int i = 0; i < ND; ++i) acc[i] *= corr;
    m = m_new;
    const int nkeys = min(32, T_total - base);
    for (int j = 0; j < nkeys; ++j) {
      const float pj = __shfl_sync(0xffffffffu, p, j);
      const T* vp = token_key(a, b, h, base + j, past, true);
      if (!vp) continue;
#pragma unroll
      for (int i = 0; i < ND; ++i) {
        const int d = lane + 32 * i;
        if (d < D) acc[i] += pj * to_float(vp[d]);
      }
    }
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  T* op = a.out + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + (int64_t)qi * a.o_sq;
#pragma unroll
  for (int i = 0; i < ND; ++i) {
    const int d = lane + 32 * i;
    if (d < D) op[d] = from_float<T>(acc[i] * inv);
  }
}

// ---------------------------------------------------------------------------
// Tensor-core readout: bf16, head width 32, no current token, no shared prefix.
// ---------------------------------------------------------------------------
constexpr int RO_TILE = 64;       // keys per shared-memory tile
constexpr int RO_PAD = 40;        // bf16 elements per staged (key, head) row, padded layout
constexpr int RO_ROW = 32;        // the same row unpadded, 16-byte pieces swizzled
constexpr int RO_WARPS = 8;

__device__ __forceinline__ void mma_bf16_16816(float c[4], const uint32_t a[4],
                                               const uint32_t b[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_bf16_raw(__nv_bfloat16 lo, __nv_bfloat16 hi) {
  __nv_bfloat162 v; v.x = lo; v.y = hi;
  return *reinterpret_cast<uint32_t*>(&v);
}

struct ReadoutArgs {
  const __nv_bfloat16* q; int64_t q_sb, q_sh, q_sq;
  const __nv_bfloat16* kc; const __nv_bfloat16* vc; int64_t kc_sp, kc_st, kc_sh;
  const int32_t* bt; int64_t bt_s; const int32_t* lengths; int num_pages;
  __nv_bfloat16* out; int64_t o_sb, o_sh, o_sq;
  int B, H, Q, page; float scale_log2;
};

// Scores, online-softmax update and P.V for one 16-query x 64-key tile of one
// head.  `valid` keys of the staged tile are real; the rest are masked.
__device__ __forceinline__ void readout_tile(const ReadoutArgs& a, int b, int h, int q0,
                                             const __nv_bfloat16* ks, const __nv_bfloat16* vs,
                                             int valid, float o[4][4], float mrow[2],
                                             float lrow[2], int g, int tig) {
  uint32_t qa[2][4];
  const __nv_bfloat16* qb = a.q + (int64_t)b * a.q_sb + (int64_t)h * a.q_sh;
  const int r0 = q0 + g, r1 = q0 + g + 8;
#pragma unroll
  for (int kq = 0; kq < 2; ++kq) {
    const int c = kq * 16 + tig * 2;
    qa[kq][0] = r0 < a.Q ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)r0 * a.q_sq + c) : 0u;
    qa[kq][1] = r1 < a.Q ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)r1 * a.q_sq + c) : 0u;
    qa[kq][2] = r0 < a.Q ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)r0 * a.q_sq + c + 8) : 0u;
    qa[kq][3] = r1 < a.Q ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)r1 * a.q_sq + c + 8) : 0u;
  }
  float s[8][4];
  const __nv_bfloat16* kh = ks + (size_t)h * RO_TILE * RO_PAD;
#pragma unroll
  for (int nb = 0; nb < 8; ++nb) {
    s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
#pragma unroll
    for (int kq = 0; kq < 2; ++kq) {
      const __nv_bfloat16* kr = kh + (size_t)(nb * 8 + g) * RO_PAD + kq * 16 + tig * 2;
      uint32_t bf[2];
      bf[0] = *reinterpret_cast<const uint32_t*>(kr);
      bf[1] = *reinterpret_cast<const uint32_t*>(kr + 8);
      mma_bf16_16816(s[nb], qa[kq], bf);
    }
  }
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const bool ok = nb * 8 + tig * 2 + c < valid;
      s[nb][c] = ok ? s[nb][c] * a.scale_log2 : -INFINITY;
      s[nb][2 + c] = ok ? s[nb][2 + c] * a.scale_log2 : -INFINITY;
      mx0 = fmaxf(mx0, s[nb][c]);
      mx1 = fmaxf(mx1, s[nb][2 + c]);
    }
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  const float mn0 = fmaxf(mrow[0], mx0), mn1 = fmaxf(mrow[1], mx1);
  const float c0 = mrow[0] == -INFINITY ? 0.f : exp2f(mrow[0] - mn0);
  const float c1 = mrow[1] == -INFINITY ? 0.f : exp2f(mrow[1] - mn1);
  float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
  for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      s[nb][c] = s[nb][c] == -INFINITY ? 0.f : exp2f(s[nb][c] - mn0);
      s[nb][2 + c] = s[nb][2 + c] == -INFINITY ? 0.f : exp2f(s[nb][2 + c] - mn1);
      sum0 += s[nb][c];
      sum1 += s[nb][2 + c];
    }
  }
  sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
  sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
  sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
  sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
  lrow[0] = lrow[0] * c0 + sum0;
  lrow[1] = lrow[1] * c1 + sum1;
  mrow[0] = mn0; mrow[1] = mn1;
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    o[n][0] *= c0; o[n][1] *= c0; o[n][2] *= c1; o[n][3] *= c1;
  }
  const __nv_bfloat16* vh = vs + (size_t)h * RO_TILE * RO_PAD;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t pa[4];
    pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
    pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
    pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
    pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
      const int key0 = kk * 16 + tig * 2;
      const int dim = nb * 8 + g;
      uint32_t bf[2];
      bf[0] = pack_bf16_raw(vh[(size_t)key0 * RO_PAD + dim], vh[(size_t)(key0 + 1) * RO_PAD + dim]);
      bf[1] = pack_bf16_raw(vh[(size_t)(key0 + 8) * RO_PAD + dim], vh[(size_t)(key0 + 9) * RO_PAD + dim]);
      mma_bf16_16816(o[nb], pa, bf);
    }
  }
}

__device__ __forceinline__ void readout_store(const ReadoutArgs& a, int b, int h, int q0,
                                              const float o[4][4], const float lrow[2],
                                              int g, int tig) {
  const float inv0 = lrow[0] > 0.f ? 1.f / lrow[0] : 0.f;
  const float inv1 = lrow[1] > 0.f ? 1.f / lrow[1] : 0.f;
  __nv_bfloat16* ob = a.out + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh;
  const int r0 = q0 + g, r1 = q0 + g + 8;
#pragma unroll
  for (int nb = 0; nb < 4; ++nb) {
    const int c = nb * 8 + tig * 2;
    if (r0 < a.Q)
      *reinterpret_cast<uint32_t*>(ob + (int64_t)r0 * a.o_sq + c) =
          pack_bf16(o[nb][0] * inv0, o[nb][1] * inv0);
    if (r1 < a.Q)
      *reinterpret_cast<uint32_t*>(ob + (int64_t)r1 * a.o_sq + c) =
          pack_bf16(o[nb][2] * inv1, o[nb][3] * inv1);
  }
}

// Stage keys/values [t0, t0 + 64) of every head of beam b (16-byte vectors).
// kSwizzled: 64-byte rows whose 16-byte piece v sits at v ^ ((t >> 1) & 3),
// so the 8 rows an ldmatrix reads cover all 32 banks without padding;
// otherwise rows padded to RO_PAD elements.
template <bool kSwizzled>
__device__ __forceinline__ void readout_stage(const ReadoutArgs& a, int b, int t0, int length,
                                              __nv_bfloat16* ks, __nv_bfloat16* vs) {
  const int total_vec = RO_TILE * a.H * 4;
  for (int idx = threadIdx.x; idx < total_vec; idx += blockDim.x) {
    const int v = idx & 3;
    const int h = (idx >> 2) % a.H;
    const int t = idx / (4 * a.H);
    const int tok = t0 + t;
    uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
    const int page = tok < length ? a.bt[(int64_t)b * a.bt_s + tok / a.page] : -1;
    if (page >= 0 && page < a.num_pages) {
      const int64_t off = (int64_t)page * a.kc_sp + (int64_t)(tok % a.page) * a.kc_st +
                          (int64_t)h * a.kc_sh + v * 8;
      kv = __ldg(reinterpret_cast<const uint4*>(a.kc + off));
      vv = __ldg(reinterpret_cast<const uint4*>(a.vc + off));
    }
    const size_t soff = kSwizzled ? ((size_t)h * RO_TILE + t) * RO_ROW + ((v ^ ((t >> 1) & 3)) * 8)
                                  : ((size_t)h * RO_TILE + t) * RO_PAD + v * 8;
    *reinterpret_cast<uint4*>(ks + soff) = kv;
    *reinterpret_cast<uint4*>(vs + soff) = vv;
  }
}

// The query fragments of one task (16 queries of head h from q0): rows
// past Q read as zeros
__device__ __forceinline__ void readout_load_q(const ReadoutArgs& a, int b, int h, int q0, int g,
                                               int tig, uint32_t qa[2][4]) {
  const __nv_bfloat16* qb = a.q + (int64_t)b * a.q_sb + (int64_t)h * a.q_sh;
  const int r0 = q0 + g, r1 = q0 + g + 8;
#pragma unroll
  for (int kq = 0; kq < 2; ++kq) {
    const int c = kq * 16 + tig * 2;
    qa[kq][0] = r0 < a.Q ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)r0 * a.q_sq + c) : 0u;
    qa[kq][1] = r1 < a.Q ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)r1 * a.q_sq + c) : 0u;
    qa[kq][2] = r0 < a.Q ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)r0 * a.q_sq + c + 8) : 0u;
    qa[kq][3] = r1 < a.Q ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)r1 * a.q_sq + c + 8) : 0u;
  }
}

__device__ __forceinline__ void ro_ldsm_x4(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((unsigned)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ro_ldsm_x4_trans(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((unsigned)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ float ro_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// readout_tile for one staged tile (swizzled layout) with the query
// fragments already loaded: K fragments by ldmatrix, V fragments by
// ldmatrix.trans (both conflict-free through the piece swizzle), key blocks
// past `valid` skipped, exponentials on the hardware ex2 (the probabilities
// are rounded to bf16 for the value product)
__device__ __forceinline__ void readout_tile_q(const ReadoutArgs& a, int h, const uint32_t qa[2][4],
                                               const __nv_bfloat16* ks, const __nv_bfloat16* vs,
                                               int valid, float o[4][4], float lrow[2], int lane) {
  const int g = lane >> 2, tig = lane & 3, mi = lane >> 3, ri = lane & 7;
  const __nv_bfloat16* kh = ks + (size_t)h * RO_TILE * RO_ROW;
  const __nv_bfloat16* vh = vs + (size_t)h * RO_TILE * RO_ROW;
  const int sw = (ri >> 1) & 3;                   // piece swizzle of this lane's rows
  const int nblocks = (valid + 7) / 8;            // 8-key blocks holding valid keys
  float s[8][4];
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int nb = 0; nb < 8; ++nb) {
    s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = -INFINITY;
    if (nb < nblocks) {
      // keys nb*8 .. +7; matrices: dims 0-7, 8-15, 16-23, 24-31
      uint32_t kf[4];
      ro_ldsm_x4(kf, kh + (size_t)(nb * 8 + ri) * RO_ROW + ((mi ^ sw) * 8));
      float c[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t b0[2] = {kf[0], kf[1]}, b1[2] = {kf[2], kf[3]};
      mma_bf16_16816(c, qa[0], b0);
      mma_bf16_16816(c, qa[1], b1);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool ok = nb * 8 + tig * 2 + e < valid;
        s[nb][e] = ok ? c[e] * a.scale_log2 : -INFINITY;
        s[nb][2 + e] = ok ? c[2 + e] * a.scale_log2 : -INFINITY;
      }
      mx0 = fmaxf(mx0, fmaxf(s[nb][0], s[nb][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nb][2], s[nb][3]));
    }
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  const float e0 = mx0 == -INFINITY ? 0.f : mx0, e1 = mx1 == -INFINITY ? 0.f : mx1;
  float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
  for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      s[nb][e] = ro_exp2(s[nb][e] - e0);
      s[nb][2 + e] = ro_exp2(s[nb][2 + e] - e1);
      sum0 += s[nb][e];
      sum1 += s[nb][2 + e];
    }
  }
  sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
  sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
  sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
  sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
  lrow[0] = sum0;
  lrow[1] = sum1;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    if (2 * kk < nblocks) {
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        // matrices: keys kk*16 + 0-7 / 8-15, dims (2 np) * 8 and (2 np + 1) * 8
        uint32_t vf[4];
        ro_ldsm_x4_trans(vf, vh + (size_t)(kk * 16 + (mi & 1) * 8 + ri) * RO_ROW +
                                 (((2 * np + (mi >> 1)) ^ sw) * 8));
        const uint32_t b0[2] = {vf[0], vf[1]}, b1[2] = {vf[2], vf[3]};
        mma_bf16_16816(o[2 * np], pa, b0);
        mma_bf16_16816(o[2 * np + 1], pa, b1);
      }
    }
  }
}

// Histories of at most 64 tokens: one staged tile serves every task; each
// warp loads its next task's queries while it computes the current one.
__global__ void __launch_bounds__(RO_WARPS * 32) readout_single_tile_kernel(ReadoutArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* vs = ks + (size_t)a.H * RO_TILE * RO_ROW;
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int length = min(a.lengths[b], RO_TILE);
  const int tasks = ((a.Q + 15) / 16) * a.H;
  if (length > 0) {
    readout_stage<true>(a, b, 0, length, ks, vs);
    __syncthreads();
  }
  uint32_t qn[2][4] = {};
  if (warp < tasks && length > 0) readout_load_q(a, b, warp % a.H, (warp / a.H) * 16, g, tig, qn);
  for (int task = warp; task < tasks; task += RO_WARPS) {
    const int h = task % a.H, q0 = (task / a.H) * 16;
    uint32_t qa[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) qa[i][j] = qn[i][j];
    const int next = task + RO_WARPS;
    if (next < tasks && length > 0)
      readout_load_q(a, b, next % a.H, (next / a.H) * 16, g, tig, qn);
    float o[4][4] = {};
    float lrow[2] = {0.f, 0.f};
    if (length > 0) readout_tile_q(a, h, qa, ks, vs, length, o, lrow, lane);
    readout_store(a, b, h, q0, o, lrow, g, tig);
  }
}

// Longer histories: each warp keeps MAXT tasks' accumulators while the CTA
// walks the key tiles.
template <int MAXT>
__global__ void __launch_bounds__(RO_WARPS * 32) readout_multi_tile_kernel(ReadoutArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* vs = ks + (size_t)a.H * RO_TILE * RO_PAD;
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int length = a.lengths[b];
  const int tasks = ((a.Q + 15) / 16) * a.H;
  const int per_warp = (tasks + RO_WARPS - 1) / RO_WARPS;
  for (int chunk = 0; chunk < per_warp; chunk += MAXT) {
    float o[MAXT][4][4] = {};
    float mrow[MAXT][2], lrow[MAXT][2];
#pragma unroll
    for (int i = 0; i < MAXT; ++i) {
      mrow[i][0] = mrow[i][1] = -INFINITY; lrow[i][0] = lrow[i][1] = 0.f;
    }
    for (int t0 = 0; t0 < length; t0 += RO_TILE) {
      __syncthreads();
      readout_stage<false>(a, b, t0, length, ks, vs);
      __syncthreads();
#pragma unroll
      for (int i = 0; i < MAXT; ++i) {
        const int task = warp + (chunk + i) * RO_WARPS;
        if (task < tasks)
          readout_tile(a, b, task % a.H, (task / a.H) * 16, ks, vs, min(RO_TILE, length - t0),
                       o[i], mrow[i], lrow[i], g, tig);
      }
    }
#pragma unroll
    for (int i = 0; i < MAXT; ++i) {
      const int task = warp + (chunk + i) * RO_WARPS;
      if (task < tasks) readout_store(a, b, task % a.H, (task / a.H) * 16, o[i], lrow[i], g, tig);
    }
  }
}

template <typename T, int D>
int launch_rows(const RowsArgs<T, D>& a, cudaStream_t stream) {
  const long long rows = (long long)a.B * a.H * a.Q;
  if (rows == 0) return GRS_OK;
  const int warps = 8;
  paged_attention_rows_kernel<T, D><<<ceil_div(rows, warps), warps * 32, 0, grs::counted(stream)>>>(a);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

template <typename T>
int dispatch_rows(int D, const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sq,
                  const void* kc, const void* vc, int64_t kc_sp, int64_t kc_st, int64_t kc_sh,
                  const int32_t* bt, int64_t bt_s, const int32_t* lengths, int num_pages,
                  const void* ck, const void* cv, int64_t ck_sb, int64_t ck_sh,
                  const uint8_t* cvalid, const void* sk, const void* sv, int num_shared,
                  void* out, int64_t o_sb, int64_t o_sh, int64_t o_sq,
                  int B, int H, int Q, int page, cudaStream_t stream) {
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)D);
#define GRS_ROWS_CASE(DD)                                                                   \
  case DD: {                                                                                \
    RowsArgs<T, DD> a{(const T*)q, q_sb, q_sh, q_sq, (const T*)kc, (const T*)vc, kc_sp,     \
                      kc_st, kc_sh, bt, bt_s, lengths, num_pages, (const T*)ck, (const T*)cv, ck_sb, \
                      ck_sh, cvalid, (const T*)sk, (const T*)sv, num_shared, (T*)out, o_sb, \
                      o_sh, o_sq, B, H, Q, page, scale_log2};                               \
    return launch_rows<T, DD>(a, stream);                                                   \
  }
  switch (D) {
    GRS_ROWS_CASE(4)
    GRS_ROWS_CASE(8)
    GRS_ROWS_CASE(16)
    GRS_ROWS_CASE(32)
    GRS_ROWS_CASE(64)
    GRS_ROWS_CASE(128)
    default: return GRS_ERR_SHAPE;
  }
#undef GRS_ROWS_CASE
}

}  // namespace grs

using namespace grs;

extern "C" int grs_paged_attention(
    int dtype, const void* query, int64_t q_sb, int64_t q_sh, int64_t q_sq,
    const void* key_cache, const void* value_cache, int64_t kc_sp, int64_t kc_st, int64_t kc_sh,
    const int32_t* block_table, int64_t bt_stride, const int32_t* lengths,
    const void* current_key, const void* current_value, int64_t ck_sb, int64_t ck_sh,
    const uint8_t* current_valid, const void* shared_key, const void* shared_value,
    int64_t num_shared, void* output, int64_t o_sb, int64_t o_sh, int64_t o_sq, int batch,
    int heads, int query_len, int head_width, int page_size, int max_blocks, int num_pages,
    void* stream_ptr) {
  cudaStream_t stream = (cudaStream_t)stream_ptr;
  if (batch < 0 || heads <= 0 || query_len < 0 || page_size <= 0 || num_shared < 0)
    return GRS_ERR_SHAPE;
  if ((current_key == nullptr) != (current_value == nullptr) ||
      (current_key == nullptr) != (current_valid == nullptr))
    return GRS_ERR_SHAPE;
  if (dtype == GRS_DTYPE_BF16 && head_width == 32 && current_key == nullptr &&
      shared_key == nullptr && query_len >= 16 && q_sq % 2 == 0 && o_sq % 2 == 0 &&
      kc_sh % 8 == 0 && kc_st % 8 == 0 && kc_sp % 8 == 0 &&
      ((uintptr_t)key_cache % 16) == 0 && ((uintptr_t)value_cache % 16) == 0 &&
      ((uintptr_t)query % 4) == 0 && ((uintptr_t)output % 4) == 0 && heads <= 16) {
    if (batch == 0) return GRS_OK;
    ReadoutArgs a{(const __nv_bfloat16*)query, q_sb, q_sh, q_sq,
                  (const __nv_bfloat16*)key_cache, (const __nv_bfloat16*)value_cache,
                  kc_sp, kc_st, kc_sh, block_table, bt_stride, lengths, num_pages,
                  (__nv_bfloat16*)output, o_sb, o_sh, o_sq, batch, heads, query_len,
                  page_size, 1.4426950408889634f / sqrtf(32.f)};
    // the single-tile kernel stages unpadded swizzled rows (64 KB at 8
    // heads: three CTAs per SM), the multi-tile kernel padded ones
    const size_t smem_single = (size_t)2 * heads * RO_TILE * RO_ROW * sizeof(__nv_bfloat16);
    const size_t smem = (size_t)2 * heads * RO_TILE * RO_PAD * sizeof(__nv_bfloat16);
    int dev = 0;
    cudaGetDevice(&dev);
    static bool attr_set[64] = {};
    if (dev < 64 && !attr_set[dev]) {
      cudaFuncSetAttribute(readout_single_tile_kernel,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
      cudaFuncSetAttribute(readout_multi_tile_kernel<4>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
      attr_set[dev] = true;
    }
    if ((int64_t)max_blocks * page_size <= RO_TILE)
      readout_single_tile_kernel<<<batch, RO_WARPS * 32, smem_single, grs::counted(stream)>>>(a);
    else
      readout_multi_tile_kernel<4><<<batch, RO_WARPS * 32, smem, grs::counted(stream)>>>(a);
    GRS_CUDA_CHECK_LAUNCH();
    return GRS_OK;
  }
  if (dtype == GRS_DTYPE_BF16)
    return dispatch_rows<__nv_bfloat16>(head_width, query, q_sb, q_sh, q_sq, key_cache,
                                        value_cache, kc_sp, kc_st, kc_sh, block_table,
                                        bt_stride, lengths, num_pages, current_key,
                                        current_value, ck_sb,
                                        ck_sh, current_valid, shared_key, shared_value,
                                        (int)num_shared, output, o_sb, o_sh, o_sq, batch,
                                        heads, query_len, page_size, stream);
  if (dtype == GRS_DTYPE_F32)
    return dispatch_rows<float>(head_width, query, q_sb, q_sh, q_sq, key_cache, value_cache,
                                kc_sp, kc_st, kc_sh, block_table, bt_stride, lengths,
                                num_pages, current_key, current_value, ck_sb, ck_sh,
                                current_valid,
                                shared_key, shared_value, (int)num_shared, output, o_sb,
                                o_sh, o_sq, batch, heads, query_len, page_size, stream);
  return GRS_ERR_SHAPE;
}
