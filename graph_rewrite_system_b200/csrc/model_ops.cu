// Row-wise fused kernels of the paged action model (reference paged_model.py,
// model.py).  The projections are the tensor-core GEMMs of gemm_tc.cu (fp32
// path: cuBLAS); every other operation of the one-token step, the node
// readout and the readout graph is one of the kernels below.  Each kernel is
// templated on the activation type (fp32 for the CPU-equivalence
// configuration, bf16 for the rollout) and computes in fp32.  Rows are processed one warp per row; each lane owns the
// row elements lane, lane + 32, ... (coalesced 32-lane accesses).
#include <algorithm>
#include <type_traits>

#include "grs_common.cuh"

namespace grs {

// GELU(x) = x/2 (1 + erf(x / sqrt 2)) (the reference's exact, erf-based
// form).  erfc comes from Abramowitz & Stegun, Handbook of Mathematical
// Functions (1964), eq. 7.1.28: for z >= 0, erf(z) = 1 - (1 + a1 z + ... +
// a6 z^6)^-16 + e(z) with |e(z)| <= 3e-7 (about 1e-6 after fp32 rounding);
// x < 0 uses erfc directly (1 + erf(-z) = erfc(z)), so nothing cancels.  One
// hardware reciprocal and ten multiply-adds per element (z is clamped at 5,
// where erfc(5) = 1.5e-12 is below fp32 resolution next to 1), so the
// elementwise kernels that apply it stay close to bandwidth-bound.
__device__ __forceinline__ float gelu_exact(float x) {
  const float z = fminf(fabsf(x) * 0.70710678118654752f, 5.f);
  float q = fmaf(0.0000430638f, z, 0.0002765672f);
  q = fmaf(q, z, 0.0001520143f);
  q = fmaf(q, z, 0.0092705272f);
  q = fmaf(q, z, 0.0422820123f);
  q = fmaf(q, z, 0.0705230784f);
  q = fmaf(q, z, 1.f);
  q *= q;
  q *= q;
  q *= q;
  q *= q;
  const float erfc_z = __fdividef(1.f, q);
  return x >= 0.f ? x * fmaf(-0.5f, erfc_z, 1.f) : 0.5f * x * erfc_z;
}

// Two lanes of gelu_exact with the packed fp32x2 multiply-adds of sm_100
// (same operations and rounding per element, half the instructions).
__device__ __forceinline__ float2 gelu_exact2(float2 x) {
  const float2 z = make_float2(fminf(fabsf(x.x) * 0.70710678118654752f, 5.f),
                               fminf(fabsf(x.y) * 0.70710678118654752f, 5.f));
  const auto c = [](float v) { return make_float2(v, v); };
  float2 q = __ffma2_rn(c(0.0000430638f), z, c(0.0002765672f));
  q = __ffma2_rn(q, z, c(0.0001520143f));
  q = __ffma2_rn(q, z, c(0.0092705272f));
  q = __ffma2_rn(q, z, c(0.0422820123f));
  q = __ffma2_rn(q, z, c(0.0705230784f));
  q = __ffma2_rn(q, z, c(1.f));
  q = __fmul2_rn(q, q);
  q = __fmul2_rn(q, q);
  q = __fmul2_rn(q, q);
  q = __fmul2_rn(q, q);
  // h = erfc(z) / 2 (exact halving); Phi(x) = 1 - h for x >= 0, h below:
  // the same roundings as x (1 - erfc / 2) and (x / 2) erfc, on pairs
  const float2 h = __fmul2_rn(make_float2(__fdividef(1.f, q.x), __fdividef(1.f, q.y)), c(0.5f));
  const float2 om = __ffma2_rn(h, c(-1.f), c(1.f));
  return __fmul2_rn(x, make_float2(x.x >= 0.f ? om.x : h.x, x.y >= 0.f ? om.y : h.y));
}

template <int N>
__device__ __forceinline__ void gelu_inplace(float* v) {
#pragma unroll
  for (int j = 0; j + 1 < N; j += 2) {
    const float2 g = gelu_exact2(make_float2(v[j], v[j + 1]));
    v[j] = g.x;
    v[j + 1] = g.y;
  }
  if (N % 2) v[N - 1] = gelu_exact(v[N - 1]);
}

template <typename T> struct DT;
template <> struct DT<float> { static constexpr int code = GRS_DTYPE_F32; };
template <> struct DT<__nv_bfloat16> { static constexpr int code = GRS_DTYPE_BF16; };

constexpr int ROW_WARPS = 8;  // rows per CTA

// ---------------------------------------------------------------------------
// s = x + scale[row] * y;   (y, scale optional)
// zc = zero_row[row] && zero_beam[beam];   wc = where_row && where_beam && where_len > 0
// if zero_before: s = zc ? s : 0
// sum_out = s
// r = wc ? LN(s) : x;  if !zero_before: r = zc ? r : 0;   ln_out = r
// beam = row / rows_per_beam.  Null masks are true.
// ---------------------------------------------------------------------------
struct AddLnArgs {
  const void* x; int64_t x_stride;
  const void* y; int64_t y_stride;
  const float* scale;
  const float* gamma; const float* beta;
  void* sum_out; int64_t sum_stride;
  void* ln_out; int64_t ln_stride;
  const uint8_t* zero_row; const uint8_t* zero_beam;
  const uint8_t* where_row; const uint8_t* where_beam; const int32_t* where_len;
  int64_t rows; int rows_per_beam; int width; float eps; int zero_before;
};

template <typename T, int VPL>
__global__ void __launch_bounds__(ROW_WARPS * 32) add_ln_kernel(AddLnArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * ROW_WARPS + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const int64_t beam = row / a.rows_per_beam;
  const T* x = reinterpret_cast<const T*>(a.x) + row * a.x_stride;
  const T* y = a.y ? reinterpret_cast<const T*>(a.y) + row * a.y_stride : nullptr;
  const float sc = a.scale ? a.scale[row] : 1.f;
  bool zc = true, wc = true;
  if (a.zero_row) zc = zc && a.zero_row[row];
  if (a.zero_beam) zc = zc && a.zero_beam[beam];
  if (a.where_row) wc = wc && a.where_row[row];
  if (a.where_beam) wc = wc && a.where_beam[beam];
  if (a.where_len) wc = wc && a.where_len[beam] > 0;
  float xv[VPL], s[VPL];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int i = lane + 32 * j;
    xv[j] = 0.f; s[j] = 0.f;
    if (i < a.width) {
      xv[j] = to_float(x[i]);
      s[j] = xv[j] + (y ? sc * to_float(y[i]) : 0.f);
      if (a.zero_before && !zc) s[j] = 0.f;
      sum += s[j];
    }
  }
  if (a.sum_out) {
    T* so = reinterpret_cast<T*>(a.sum_out) + row * a.sum_stride;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int i = lane + 32 * j;
      if (i < a.width) so[i] = from_float<T>(s[j]);
    }
  }
  if (!a.ln_out) return;
  const float mean = warp_sum(sum) / a.width;
  float var = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int i = lane + 32 * j;
    if (i < a.width) { const float d = s[j] - mean; var += d * d; }
  }
  const float rstd = rsqrtf(warp_sum(var) / a.width + a.eps);
  T* lo = reinterpret_cast<T*>(a.ln_out) + row * a.ln_stride;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int i = lane + 32 * j;
    if (i < a.width) {
      float r = wc ? (s[j] - mean) * rstd * a.gamma[i] + a.beta[i] : xv[j];
      if (!a.zero_before && !zc) r = 0.f;
      lo[i] = from_float<T>(r);
    }
  }
}

// Eight consecutive elements as fp32, loaded/stored with 16-byte (bf16) or
// 2 x 16-byte (fp32) accesses; the pointer must be aligned to that width.
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float v[8]) {
  const uint4 x = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float v[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
// R 16-byte pieces of 8 bf16 each into 8 R floats
template <int R>
__device__ __forceinline__ void unpack_bf16x8(const uint4 (&r)[R], float* v) {
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      v[8 * i + 2 * j] = f.x;
      v[8 * i + 2 * j + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float v[8]) {
  uint4 x;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&x);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
  *reinterpret_cast<uint4*>(p) = x;
}
__device__ __forceinline__ void store8(float* p, const float v[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// In place: y[r, c] = GELU(y[r, c] + bias[c]) (bias optional).  Each thread
// handles groups of 8 consecutive columns (cols % 8 == 0, 16-byte aligned
// rows), grid-strided.
template <typename T, typename I>
__global__ void bias_gelu_kernel(T* y, int64_t rows, int cols, int64_t stride,
                                 const float* bias, int apply_gelu) {
  const I groups = (I)(cols >> 3);
  const I n = (I)rows * groups;   // I = uint32_t whenever the group count fits
  for (I g = (I)blockIdx.x * blockDim.x + threadIdx.x; g < n; g += (I)gridDim.x * blockDim.x) {
    const I r = g / groups;
    const int c = (int)(g - r * groups) << 3;
    T* p = y + r * stride + c;
    float v[8];
    load8(p, v);
    if (bias) {
      float b[8];
      load8(bias + c, b);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += b[j];
    }
    if (apply_gelu) gelu_inplace<8>(v);
    store8(p, v);
  }
}

// states[b, s] = (gate_embedding[max(type, 0)] + marker) * (type >= 0)
// (paged_model.py:246-250); live[b, s] = type >= 0.
template <typename T>
__global__ void embed_initial_kernel(const int64_t* types, int64_t rows, int width,
                                     const float* gate_emb, const float* marker, T* states,
                                     int64_t stride, uint8_t* live) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * ROW_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t t = types[row];
  if (lane == 0) live[row] = t >= 0;
  const float* e = gate_emb + (t < 0 ? 0 : t) * width;
  for (int i = lane; i < width; i += 32)
    states[row * stride + i] = from_float<T>(t >= 0 ? e[i] + marker[i] : 0.f);
}

// Message-passing aggregation of InitialGraphLayer (model.py:36-51) over the
// port arrays: each node gathers forward messages from its in-ports and
// backward messages from its out-ports, adds the relation embeddings and
// divides by its degree.  No atomics: the port arrays are the CSR.
//   fb [B*S, 2W]: forward_message(x) | backward_message(x); rel [32, W] (fp32)
//   ports [B, S, 4] int32 each; out writes agg into agg [B*S] rows (stride).
template <typename T, int VPL>
__global__ void __launch_bounds__(ROW_WARPS * 32) graph_aggregate_kernel(
    const T* fb, int64_t fb_stride, const float* rel, const int32_t* in_node,
    const int32_t* in_port, const int32_t* out_node, const int32_t* out_port, int64_t rows,
    int slots, int port_slots, int width, T* agg, int64_t agg_stride) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * ROW_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t beam_base = (row / slots) * slots;
  const int64_t prow = (row / slots) * port_slots + row % slots;
  float acc[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) acc[j] = 0.f;
  int deg = 0;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const int src = in_node[prow * 4 + p];
    if (src >= 0) {
      const int r = in_port[prow * 4 + p] * 4 + p;
      const T* f = fb + (beam_base + src) * fb_stride;
      const float* e = rel + (int64_t)r * width;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int i = lane + 32 * j;
        if (i < width) acc[j] += to_float(f[i]) + e[i];
      }
      ++deg;
    }
    const int dst = out_node[prow * 4 + p];
    if (dst >= 0) {
      const int r = 16 + p * 4 + out_port[prow * 4 + p];
      const T* bk = fb + (beam_base + dst) * fb_stride + width;
      const float* e = rel + (int64_t)r * width;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int i = lane + 32 * j;
        if (i < width) acc[j] += to_float(bk[i]) + e[i];
      }
      ++deg;
    }
  }
  const float inv = 1.f / (float)(deg > 0 ? deg : 1);
  T* o = agg + row * agg_stride;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int i = lane + 32 * j;
    if (i < width) o[i] = from_float<T>(acc[j] * inv);
  }
}

// Action inputs (paged_model.py:502-523): bound[b, k] = states[b, max(slot,0)],
// source_mask[b, k] = slot >= 0 && active; ctx_in[b] = [xfer_emb[max(x,0)],
// source_reps[max(s,0)], mean of bound over the mask]; active[b] = x >= 0.
template <typename T>
__global__ void action_inputs_kernel(const T* states, int64_t state_stride, int slots,
                                     const int64_t* xfer_ids, const int64_t* source_ids,
                                     const int64_t* source_slots, int pattern, int width,
                                     const float* xfer_emb, const float* source_reps, T* bound,
                                     T* ctx_in, uint8_t* source_mask, uint8_t* active, int batch) {
  const int b = blockIdx.x;
  if (b >= batch) return;
  const int64_t x = xfer_ids[b];
  const bool act = x >= 0;
  const int64_t s = source_ids[b] < 0 ? 0 : source_ids[b];
  int count = 0;
  for (int k = 0; k < pattern; ++k) count += (source_slots[(int64_t)b * pattern + k] >= 0 && act);
  const float inv = 1.f / (float)(count > 0 ? count : 1);
  if (threadIdx.x == 0) active[b] = act;
  if (threadIdx.x < pattern) {
    const int64_t slot = source_slots[(int64_t)b * pattern + threadIdx.x];
    source_mask[(int64_t)b * pattern + threadIdx.x] = slot >= 0 && act;
  }
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    float pool = 0.f;
    for (int k = 0; k < pattern; ++k) {
      const int64_t slot = source_slots[(int64_t)b * pattern + k];
      const int64_t safe = slot < 0 ? 0 : slot;
      const T v = states[((int64_t)b * slots + safe) * state_stride + i];
      bound[((int64_t)b * pattern + k) * width + i] = v;
      if (slot >= 0 && act) pool += to_float(v);
    }
    T* c = ctx_in + (int64_t)b * 3 * width;
    c[i] = from_float<T>(xfer_emb[(x < 0 ? 0 : x) * width + i]);
    c[width + i] = from_float<T>(source_reps[s * width + i]);
    c[2 * width + i] = from_float<T>(pool * inv);
  }
}

// token[b] = (raw[b] + position[len[b]]) * active[b]   (paged_model.py:524-525)
template <typename T>
__global__ void position_token_kernel(const T* raw, const float* position, const int32_t* lengths,
                                      const uint8_t* active, T* token, int batch, int width) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)batch * width) return;
  const int b = (int)(idx / width), i = (int)(idx % width);
  const float v = active[b] ? to_float(raw[idx]) + position[(int64_t)lengths[b] * width + i] : 0.f;
  token[idx] = from_float<T>(v);
}

// N consecutive elements as fp32 with the widest aligned accesses (the
// pointer must be aligned to min(16, N * sizeof(T)) bytes).
template <int N>
__device__ __forceinline__ void load_vec(const __nv_bfloat16* p, float* v) {
  if constexpr (N >= 8) {
#pragma unroll
    for (int i = 0; i < N / 8; ++i) load8(p + 8 * i, v + 8 * i);
  } else if constexpr (N == 4) {
    const uint2 x = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  } else if constexpr (N == 2) {
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    v[0] = a.x; v[1] = a.y;
  } else {
    v[0] = __bfloat162float(p[0]);
  }
}
template <int N>
__device__ __forceinline__ void load_vec(const float* p, float* v) {
  if constexpr (N >= 4) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      const float4 a = reinterpret_cast<const float4*>(p)[i];
      v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
    }
  } else if constexpr (N == 2) {
    const float2 a = *reinterpret_cast<const float2*>(p);
    v[0] = a.x; v[1] = a.y;
  } else {
    v[0] = p[0];
  }
}
// load_vec through the read-only data path (ld.global.nc, cached in L1):
// for gathers whose rows other warps of the same SM read too
template <int N>
__device__ __forceinline__ void load_vec_ro(const __nv_bfloat16* p, float* v) {
  if constexpr (N >= 8) {
#pragma unroll
    for (int i = 0; i < N / 8; ++i) {
      const uint4 x = __ldg(reinterpret_cast<const uint4*>(p) + i);
      unpack_bf16x8<1>(reinterpret_cast<const uint4(&)[1]>(x), v + 8 * i);
    }
  } else if constexpr (N == 4) {
    const uint2 x = __ldg(reinterpret_cast<const uint2*>(p));
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  } else if constexpr (N == 2) {
    const float2 a = __bfloat1622float2(__ldg(reinterpret_cast<const __nv_bfloat162*>(p)));
    v[0] = a.x; v[1] = a.y;
  } else {
    v[0] = __bfloat162float(__ldg(p));
  }
}
template <int N>
__device__ __forceinline__ void load_vec_ro(const float* p, float* v) {
  if constexpr (N >= 4) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(p) + i);
      v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
    }
  } else if constexpr (N == 2) {
    const float2 a = __ldg(reinterpret_cast<const float2*>(p));
    v[0] = a.x; v[1] = a.y;
  } else {
    v[0] = __ldg(p);
  }
}
template <int N>
__device__ __forceinline__ void store_vec(__nv_bfloat16* p, const float* v) {
  if constexpr (N >= 8) {
#pragma unroll
    for (int i = 0; i < N / 8; ++i) store8(p + 8 * i, v + 8 * i);
  } else if constexpr (N == 4) {
    uint2 x;
    *reinterpret_cast<__nv_bfloat162*>(&x.x) = __floats2bfloat162_rn(v[0], v[1]);
    *reinterpret_cast<__nv_bfloat162*>(&x.y) = __floats2bfloat162_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(p) = x;
  } else if constexpr (N == 2) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v[0], v[1]);
  } else {
    p[0] = __float2bfloat16_rn(v[0]);
  }
}
template <int N>
__device__ __forceinline__ void store_vec(float* p, const float* v) {
  if constexpr (N >= 4) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i)
      reinterpret_cast<float4*>(p)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else if constexpr (N == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  } else {
    p[0] = v[0];
  }
}

constexpr int ULH_ROWS = 64;   // slot rows of one beam per CTA

// Lane-interleaved shared-memory rows for per-lane chunks of V floats (V a
// multiple of 4, row length 32 V): float4 j of lane L sits at float4 index
// j * 32 + L, so a warp's 16-byte loads of one j hit 32 consecutive float4s
// (no bank conflicts; the plain layout puts lanes V floats apart, which maps
// up to 16 lanes onto the same four banks).
template <int V>
__device__ __forceinline__ void lds_interleaved(const float* row, int lane, float* out) {
#pragma unroll
  for (int j = 0; j < V / 4; ++j) {
    const float4 f = reinterpret_cast<const float4*>(row)[j * 32 + lane];
    out[4 * j] = f.x;
    out[4 * j + 1] = f.y;
    out[4 * j + 2] = f.z;
    out[4 * j + 3] = f.w;
  }
}
// rows of 32 V elements from global memory into that layout, as fp32
template <int V, typename T>
__device__ __forceinline__ void stage_interleaved(float* dst, const T* src, int rows) {
  const int n = rows * 32 * V;
  for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) {
    const int row = i / (32 * V), e = i - row * 32 * V;
    float4 f;
    f.x = to_float(src[i]);
    f.y = to_float(src[i + 1]);
    f.z = to_float(src[i + 2]);
    f.w = to_float(src[i + 3]);
    reinterpret_cast<float4*>(dst + row * 32 * V)[((e % V) / 4) * 32 + e / V] = f;
  }
}

constexpr int AGG_ROWS = 64;   // consecutive slot rows of one graph_aggregate_vec_kernel CTA

// graph_aggregate_kernel with each lane owning VPL contiguous elements
// (width == 32 * VPL): 16-byte row accesses instead of 2-byte ones.  Every
// element accumulates the same terms in the same order, so results are
// bit-identical to the strided kernel.  kPacked: fb and agg rows are
// 2 * width apart (the model's [in | out] and [x | agg] buffers), so the row
// strides are compile-time constants.  With 16-byte lane chunks the kernel
// fits 48 registers, so five CTAs stay resident per SM.
template <typename T, int VPL, bool kPacked>
__global__ void __launch_bounds__(ROW_WARPS * 32, VPL * sizeof(T) <= 16 ? 5 : 2)
    graph_aggregate_vec_kernel(
    const T* fb, int64_t fb_stride_arg, const float* rel, const int32_t* in_node,
    const int32_t* in_port, const int32_t* out_node, const int32_t* out_port, int64_t rows,
    int slots, int port_slots, T* agg, int64_t agg_stride_arg) {
  // a CTA takes AGG_ROWS consecutive slot rows, its warps interleaved one row
  // at a time: a slot's neighbours are nearby slots of the same beam, so most
  // neighbour rows one warp gathers were just brought into this SM's L1 by
  // another (1.2x faster than spreading consecutive rows over SMs)
  constexpr int width = 32 * VPL;
  const int64_t fb_stride = kPacked ? 2 * width : fb_stride_arg;
  const int64_t agg_stride = kPacked ? 2 * width : agg_stride_arg;
  const int lane = threadIdx.x & 31;
  const int c0 = lane * VPL;
  const int64_t first = (int64_t)blockIdx.x * AGG_ROWS + (threadIdx.x >> 5);
  const int64_t last = min(rows, (int64_t)(blockIdx.x + 1) * AGG_ROWS);
  // (beam, slot) of the row: one division for the first row, then stepped
  int64_t beam = first / slots;
  int slot = (int)(first - beam * slots);
  for (int64_t row = first; row < last; row += ROW_WARPS) {
    const int64_t prow = beam * port_slots + slot;
    const int64_t beam_base = beam * slots;
    for (slot += ROW_WARPS; slot >= slots; slot -= slots) ++beam;
    const int4 inn = __ldg(reinterpret_cast<const int4*>(in_node) + prow);
    const int4 inp = __ldg(reinterpret_cast<const int4*>(in_port) + prow);
    const int4 outn = __ldg(reinterpret_cast<const int4*>(out_node) + prow);
    const int4 outp = __ldg(reinterpret_cast<const int4*>(out_port) + prow);
    const int in_n[4] = {inn.x, inn.y, inn.z, inn.w}, in_p[4] = {inp.x, inp.y, inp.z, inp.w};
    const int out_n[4] = {outn.x, outn.y, outn.z, outn.w};
    const int out_p[4] = {outp.x, outp.y, outp.z, outp.w};
    float acc[VPL];
#pragma unroll
    for (int j = 0; j < VPL; ++j) acc[j] = 0.f;
    int deg = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int src = in_n[p];
      if (src >= 0) {
        const int r = in_p[p] * 4 + p;
        float f[VPL], e[VPL];
        load_vec_ro<VPL>(fb + (beam_base + src) * fb_stride + c0, f);
        load_vec<VPL>(rel + (int64_t)r * width + c0, e);
#pragma unroll
        for (int j = 0; j < VPL; ++j) acc[j] += f[j] + e[j];
        ++deg;
      }
      const int dst = out_n[p];
      if (dst >= 0) {
        const int r = 16 + p * 4 + out_p[p];
        float f[VPL], e[VPL];
        load_vec_ro<VPL>(fb + (beam_base + dst) * fb_stride + width + c0, f);
        load_vec<VPL>(rel + (int64_t)r * width + c0, e);
#pragma unroll
        for (int j = 0; j < VPL; ++j) acc[j] += f[j] + e[j];
        ++deg;
      }
    }
    const float inv = 1.f / (float)(deg > 0 ? deg : 1);
#pragma unroll
    for (int j = 0; j < VPL; ++j) acc[j] *= inv;
    store_vec<VPL>(agg + row * agg_stride + c0, acc);
  }
}

// add_ln_kernel with each lane owning VPL contiguous elements of the row
// (width == 32 * VPL): one 16-byte access per lane and tensor instead of
// VPL 2-byte ones.  Same semantics as add_ln_kernel.
template <typename T, int VPL>
__global__ void __launch_bounds__(ROW_WARPS * 32) add_ln_vec_kernel(AddLnArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * ROW_WARPS + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const int64_t beam = row / a.rows_per_beam;
  const int c0 = lane * VPL;
  const float sc = a.scale ? a.scale[row] : 1.f;
  bool zc = true, wc = true;
  if (a.zero_row) zc = zc && a.zero_row[row];
  if (a.zero_beam) zc = zc && a.zero_beam[beam];
  if (a.where_row) wc = wc && a.where_row[row];
  if (a.where_beam) wc = wc && a.where_beam[beam];
  if (a.where_len) wc = wc && a.where_len[beam] > 0;
  float xv[VPL], s[VPL];
  load_vec<VPL>(reinterpret_cast<const T*>(a.x) + row * a.x_stride + c0, xv);
  if (a.y) {
    float yv[VPL];
    load_vec<VPL>(reinterpret_cast<const T*>(a.y) + row * a.y_stride + c0, yv);
#pragma unroll
    for (int j = 0; j < VPL; ++j) s[j] = xv[j] + sc * yv[j];
  } else {
#pragma unroll
    for (int j = 0; j < VPL; ++j) s[j] = xv[j];
  }
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    if (a.zero_before && !zc) s[j] = 0.f;
    sum += s[j];
  }
  if (a.sum_out) store_vec<VPL>(reinterpret_cast<T*>(a.sum_out) + row * a.sum_stride + c0, s);
  if (!a.ln_out) return;
  const float mean = warp_sum(sum) / a.width;
  float var = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const float d = s[j] - mean;
    var += d * d;
  }
  const float rstd = rsqrtf(warp_sum(var) / a.width + a.eps);
  float r[VPL];
  if (wc) {
    float g[VPL], b[VPL];
    load_vec<VPL>(a.gamma + c0, g);
    load_vec<VPL>(a.beta + c0, b);
#pragma unroll
    for (int j = 0; j < VPL; ++j) r[j] = (s[j] - mean) * rstd * g[j] + b[j];
  } else {
#pragma unroll
    for (int j = 0; j < VPL; ++j) r[j] = xv[j];
  }
  if (!a.zero_before && !zc) {
#pragma unroll
    for (int j = 0; j < VPL; ++j) r[j] = 0.f;
  }
  store_vec<VPL>(reinterpret_cast<T*>(a.ln_out) + row * a.ln_stride + c0, r);
}

// _update_live_nodes hidden layer (paged_model.py:223-238), per slot row:
//   logits_k = q . key[b,k] / sqrt(W) (masked -1e4), attn = softmax_k,
//   affinity = sigmoid(max_k logits),
//   h = GELU(xa + sum_k attn_k * vw[b,k] + c[b])
// with q = states W_query^T, xa = states W1[:, :W]^T (one GEMM, qxa row =
// [q | xa]), vw[b,k] = (bound W_value^T) W1[:, W:2W]^T, c[b] = ctx W1[:, 2W:]^T + b1.
// A CTA takes up to ULH_ROWS slot rows of one beam (grid = row blocks x
// beams) and stages that beam's keys, vw and c in shared memory (fp32) once;
// a warp handles a row, each lane a contiguous chunk of VPLQ (q) and VPLH
// (xa, h) elements, read and written with vector accesses.
template <typename T, int VPLQ, int VPLH>
__global__ void __launch_bounds__(ROW_WARPS * 32, 4) update_live_hidden_kernel(
    const T* qxa, int64_t qxa_stride, const T* keys, const T* vw, const T* cvec,
    const uint8_t* source_mask, int pattern, int slots, int width, T* hidden,
    int64_t hidden_stride, float* affinity, int interleave) {
  extern __shared__ __align__(16) float ulh_smem[];
  const int hw = 2 * width;
  float* ks = ulh_smem;                          // [pattern][width]
  float* vs = ks + pattern * width;              // [pattern][2W]
  float* cs = vs + pattern * hw;                 // [2W]
  __shared__ bool s_mask[8];
  const int64_t b = blockIdx.y;
  // `interleave` (width == 32 VPLQ, 2 width == 32 VPLH, both multiples of
  // 4): the lane-interleaved layout; otherwise rows as they are
  constexpr bool kCanInterleave = VPLQ % 4 == 0 && VPLH % 4 == 0;
  const bool inter = kCanInterleave && interleave;
  if (inter) {
    stage_interleaved<(kCanInterleave ? VPLQ : 4)>(ks, keys + b * pattern * width, pattern);
    stage_interleaved<(kCanInterleave ? VPLH : 4)>(vs, vw + b * pattern * hw, pattern);
    stage_interleaved<(kCanInterleave ? VPLH : 4)>(cs, cvec + b * hw, 1);
  } else {
    for (int i = threadIdx.x; i < pattern * width; i += blockDim.x)
      ks[i] = to_float(keys[b * pattern * width + i]);
    for (int i = threadIdx.x; i < pattern * hw; i += blockDim.x)
      vs[i] = to_float(vw[b * pattern * hw + i]);
    for (int i = threadIdx.x; i < hw; i += blockDim.x) cs[i] = to_float(cvec[b * hw + i]);
  }
  if (threadIdx.x < pattern) s_mask[threadIdx.x] = source_mask[b * pattern + threadIdx.x] != 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q0 = lane * VPLQ, h0 = lane * VPLH;
  const bool q_on = q0 < width, h_on = h0 < hw;
  const float scale = rsqrtf((float)width);
  const int end = min(slots, (blockIdx.x + 1) * ULH_ROWS);
  // bf16 rows in 16-byte pieces: the next row's query and input pieces are
  // requested before this row's attention, so each warp has two rows' loads
  // in flight instead of one
  constexpr bool kAhead = std::is_same<T, __nv_bfloat16>::value && VPLQ % 8 == 0 && VPLH % 8 == 0;
  constexpr int RQ = kAhead ? VPLQ / 8 : 1, RH = kAhead ? VPLH / 8 : 1;
  uint4 rq[RQ], rh[RH];
  const auto fetch = [&](int slot) {
    const T* q = qxa + (b * slots + slot) * qxa_stride;
#pragma unroll
    for (int i = 0; i < RQ; ++i)
      rq[i] = q_on ? __ldg(reinterpret_cast<const uint4*>(q + q0) + i) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < RH; ++i)
      rh[i] = h_on ? __ldg(reinterpret_cast<const uint4*>(q + width + h0) + i)
                   : make_uint4(0, 0, 0, 0);
  };
  if (kAhead && blockIdx.x * ULH_ROWS + warp < end) fetch(blockIdx.x * ULH_ROWS + warp);
  for (int s = blockIdx.x * ULH_ROWS + warp; s < end; s += ROW_WARPS) {
    const int64_t row = b * slots + s;
    float qv[VPLQ], xv[VPLH];
    if constexpr (kAhead) {
      unpack_bf16x8<RQ>(rq, qv);
      unpack_bf16x8<RH>(rh, xv);
      if (s + ROW_WARPS < end) fetch(s + ROW_WARPS);
    } else {
      const T* q = qxa + row * qxa_stride;
      if (q_on) load_vec<VPLQ>(q + q0, qv);
      else
#pragma unroll
        for (int j = 0; j < VPLQ; ++j) qv[j] = 0.f;
      if (h_on) load_vec<VPLH>(q + width + h0, xv);
    }
    float logit[8];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < 8; ++k) {   // pattern <= 8: logits stay in registers
      logit[k] = 0.f;
      if (k >= pattern) continue;
      float d = 0.f;
      if (q_on) {
        float kv[VPLQ];
        if constexpr (kCanInterleave) {
          if (inter) lds_interleaved<VPLQ>(ks + k * width, lane, kv);
          else load_vec<VPLQ>(ks + k * width + q0, kv);
        } else {
          load_vec<VPLQ>(ks + k * width + q0, kv);
        }
#pragma unroll
        for (int j = 0; j < VPLQ; ++j) d += qv[j] * kv[j];
      }
      d = warp_sum(d) * scale;
      if (!s_mask[k]) d = -1e4f;
      logit[k] = d;
      mx = fmaxf(mx, d);
    }
    float den = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k >= pattern) continue;
      logit[k] = __expf(logit[k] - mx);
      den += logit[k];
    }
    const float inv = 1.f / den;
    if (lane == 0) affinity[row] = 1.f / (1.f + __expf(-mx));
    if (h_on) {
      float acc[VPLH];
      if constexpr (kCanInterleave) {
        if (inter) lds_interleaved<VPLH>(cs, lane, acc);
        else load_vec<VPLH>(cs + h0, acc);
      } else {
        load_vec<VPLH>(cs + h0, acc);
      }
#pragma unroll
      for (int j = 0; j < VPLH; ++j) acc[j] += xv[j];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (k >= pattern) continue;
        float vv[VPLH];
        if constexpr (kCanInterleave) {
          if (inter) lds_interleaved<VPLH>(vs + k * hw, lane, vv);
          else load_vec<VPLH>(vs + k * hw + h0, vv);
        } else {
          load_vec<VPLH>(vs + k * hw + h0, vv);
        }
        const float w = logit[k] * inv;
#pragma unroll
        for (int j = 0; j < VPLH; ++j) acc[j] += w * vv[j];
      }
      gelu_inplace<VPLH>(acc);
      store_vec<VPLH>(hidden + row * hidden_stride + h0, acc);
    }
  }
}

// destination_state hidden layer (paged_model.py:592-601):
//   h[b, j] = GELU(r[b] + type_table[type] + position_table[j]) for valid
//   destinations, where r = raw W0[:, :W]^T + b0, type_table = gate_emb
//   W0[:, W:2W]^T and position_table = pattern_position W0[:, 2W:]^T.
template <typename T>
__global__ void destination_hidden_kernel(const T* r, const float* type_table,
                                          const float* pos_table, const int64_t* dest_slots,
                                          const int64_t* dest_types, const uint8_t* active,
                                          int pattern, int batch, int hw, T* hidden) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)batch * pattern * hw) return;
  const int i = (int)(idx % hw);
  const int64_t bj = idx / hw;
  const int j = (int)(bj % pattern);
  const int b = (int)(bj / pattern);
  const bool valid = dest_slots[bj] >= 0 && active[b];
  float v = 0.f;
  if (valid) {
    const int64_t t = dest_types[bj];
    v = gelu_exact(to_float(r[(int64_t)b * hw + i]) + type_table[t * hw + i] + pos_table[(int64_t)j * hw + i]);
  }
  hidden[idx] = from_float<T>(v);
}

// Kill source slots then create destination slots (paged_model.py:569-604).
template <typename T>
__global__ void apply_slots_kernel(T* states, int64_t state_stride, uint8_t* live, int64_t* types,
                                   int slots, const int64_t* source_slots,
                                   const uint8_t* source_mask, int spattern,
                                   const int64_t* dest_slots, const int64_t* dest_types,
                                   const uint8_t* active, int dpattern, const T* created,
                                   int width, int batch) {
  const int b = blockIdx.x;
  if (b >= batch) return;
  for (int k = 0; k < spattern; ++k) {
    if (!source_mask[(int64_t)b * spattern + k]) continue;
    const int64_t slot = source_slots[(int64_t)b * spattern + k];
    const int64_t row = (int64_t)b * slots + slot;
    for (int i = threadIdx.x; i < width; i += blockDim.x) states[row * state_stride + i] = from_float<T>(0.f);
    if (threadIdx.x == 0) { live[row] = 0; types[row] = -1; }
  }
  __syncthreads();
  if (!active[b]) return;
  for (int j = 0; j < dpattern; ++j) {
    const int64_t slot = dest_slots[(int64_t)b * dpattern + j];
    if (slot < 0) continue;
    const int64_t row = (int64_t)b * slots + slot;
    const T* c = created + ((int64_t)b * dpattern + j) * width;
    for (int i = threadIdx.x; i < width; i += blockDim.x) states[row * state_stride + i] = c[i];
    if (threadIdx.x == 0) { live[row] = 1; types[row] = dest_types[(int64_t)b * dpattern + j]; }
  }
}

// match_logits epilogue (model.py:382-389): logits = acc / sqrt(R) + bias,
// eligible = live && type == first_type[v], ineligible -> -1e4 (fp32 out).
template <typename T>
__global__ void match_logits_kernel(const T* acc, int64_t acc_stride, const float* source_bias,
                                    const int64_t* first_types, const uint8_t* live,
                                    const int64_t* types, int64_t rows, int num_sources,
                                    float inv_sqrt_r, float* logits, uint8_t* eligible) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * num_sources) return;
  const int64_t r = idx / num_sources;
  const int v = (int)(idx % num_sources);
  const bool e = live[r] && types[r] == first_types[v];
  eligible[idx] = e;
  logits[idx] = e ? to_float(acc[r * acc_stride + v]) * inv_sqrt_r + source_bias[v] : -1e4f;
}

// out[i] = in[index[i]] row by row; an input row of in_bytes is copied into
// an output row of out_bytes and the tail (out_bytes > in_bytes) is filled
// with fill_byte (0 for states and live flags, 0xff for -1 ids).
__global__ void gather_beams_kernel(const char* in, char* out, const int64_t* index,
                                    int64_t rows, int64_t in_bytes, int64_t out_bytes,
                                    int fill_byte) {
  const int64_t r = blockIdx.x;
  if (r >= rows) return;
  const char* s = in + index[r] * in_bytes;
  char* d = out + r * out_bytes;
  const int64_t copy = in_bytes < out_bytes ? in_bytes : out_bytes;
  if ((copy & 15) == 0 && (in_bytes & 15) == 0 && (out_bytes & 15) == 0 &&
      ((uintptr_t)in & 15) == 0 && ((uintptr_t)out & 15) == 0) {
    for (int64_t v = threadIdx.x; v < copy / 16; v += blockDim.x)
      reinterpret_cast<uint4*>(d)[v] = reinterpret_cast<const uint4*>(s)[v];
  } else {
    for (int64_t v = threadIdx.x; v < copy; v += blockDim.x) d[v] = s[v];
  }
  for (int64_t v = copy + threadIdx.x; v < out_bytes; v += blockDim.x) d[v] = (char)fill_byte;
}

// Port arrays from an edge list (model.py:402-418): relation = sp * 4 + dp.
__global__ void edges_to_ports_kernel(const int64_t* eb, const int64_t* es, const int64_t* ed,
                                      const int64_t* er, int64_t edges, int slots,
                                      int32_t* out_node, int32_t* out_port, int32_t* in_node,
                                      int32_t* in_port) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= edges) return;
  const int64_t sp = er[e] / 4, dp = er[e] % 4;
  const int64_t src = eb[e] * slots + es[e], dst = eb[e] * slots + ed[e];
  out_node[src * 4 + sp] = (int32_t)ed[e];
  out_port[src * 4 + sp] = (int32_t)dp;
  in_node[dst * 4 + dp] = (int32_t)es[e];
  in_port[dst * 4 + dp] = (int32_t)sp;
}

// ---------------------------------------------------------------------------
inline int vpl_for(int width) {
  const int v = (width + 31) / 32;
  if (v <= 1) return 1;
  if (v <= 2) return 2;
  if (v <= 4) return 4;
  if (v <= 8) return 8;
  if (v <= 16) return 16;
  if (v <= 32) return 32;
  return -1;
}

}  // namespace grs

using namespace grs;

#define GRS_VPL_SWITCH(VAR, width, ...)            \
  switch (vpl_for(width)) {                        \
    case 1: { constexpr int VAR = 1; __VA_ARGS__; break; }  \
    case 2: { constexpr int VAR = 2; __VA_ARGS__; break; }  \
    case 4: { constexpr int VAR = 4; __VA_ARGS__; break; }  \
    case 8: { constexpr int VAR = 8; __VA_ARGS__; break; }  \
    case 16: { constexpr int VAR = 16; __VA_ARGS__; break; } \
    case 32: { constexpr int VAR = 32; __VA_ARGS__; break; } \
    default: return GRS_ERR_SHAPE;                 \
  }

#define GRS_DTYPE_SWITCH(T, dtype, ...)                                   \
  if ((dtype) == GRS_DTYPE_F32) { using T = float; __VA_ARGS__; }          \
  else if ((dtype) == GRS_DTYPE_BF16) { using T = __nv_bfloat16; __VA_ARGS__; } \
  else return GRS_ERR_SHAPE;

extern "C" int grs_add_layernorm(int dtype, const void* x, int64_t x_stride, const void* y,
                                 int64_t y_stride, const float* scale, const float* gamma,
                                 const float* beta, void* sum_out, int64_t sum_stride,
                                 void* ln_out, int64_t ln_stride, const uint8_t* zero_row,
                                 const uint8_t* zero_beam, const uint8_t* where_row,
                                 const uint8_t* where_beam, const int32_t* where_len,
                                 int64_t rows, int rows_per_beam, int width, float eps,
                                 int zero_before, void* stream) {
  if (rows <= 0) return GRS_OK;
  if (rows_per_beam <= 0 || width <= 0) return GRS_ERR_SHAPE;
  AddLnArgs a{x, x_stride, y, y_stride, scale, gamma, beta, sum_out, sum_stride, ln_out,
              ln_stride, zero_row, zero_beam, where_row, where_beam, where_len, rows,
              rows_per_beam, width, eps, zero_before};
  const int grid = ceil_div(rows, ROW_WARPS);
  // contiguous per-lane vectors when the row is 32 whole vectors and every
  // pointer and stride keeps them aligned
  const int esize = dtype == GRS_DTYPE_F32 ? 4 : 2;
  const int vpl = width / 32;
  const int64_t vbytes = std::min<int64_t>(16, (int64_t)vpl * esize);
  const auto ok = [&](const void* p, int64_t stride) {
    return p == nullptr ||
           ((reinterpret_cast<uintptr_t>(p) % vbytes) == 0 && (stride * esize) % vbytes == 0);
  };
  // each lane of the vector kernel owns width / 32 columns, which must be
  // one of the chunk sizes it is instantiated for (no masked tail lanes)
  const bool vec = width % 32 == 0 && vpl >= 2 && vpl <= 16 && vpl_for(width) == vpl &&
                   ok(x, x_stride) &&
                   ok(y, y_stride) && ok(sum_out, sum_stride) && ok(ln_out, ln_stride) &&
                   (reinterpret_cast<uintptr_t>(gamma) % 16) == 0 &&
                   (reinterpret_cast<uintptr_t>(beta) % 16) == 0;
  if (vec) {
    GRS_DTYPE_SWITCH(T, dtype, GRS_VPL_SWITCH(V, width,
        add_ln_vec_kernel<T, V><<<grid, ROW_WARPS * 32, 0, grs::counted((cudaStream_t)stream)>>>(a)))
  } else {
    GRS_DTYPE_SWITCH(T, dtype, GRS_VPL_SWITCH(V, width,
        add_ln_kernel<T, V><<<grid, ROW_WARPS * 32, 0, grs::counted((cudaStream_t)stream)>>>(a)))
  }
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_bias_gelu(int dtype, void* y, int64_t rows, int cols, int64_t stride,
                             const float* bias, int apply_gelu, void* stream) {
  if (rows <= 0) return GRS_OK;
  // 8-column groups with 16-byte (bf16) / 32-byte (fp32) aligned accesses
  if (cols % 8 || stride % 8 || ((uintptr_t)y & 15) || ((uintptr_t)bias & 15)) return GRS_ERR_SHAPE;
  const int64_t groups = rows * (cols / 8);
  const int grid = (int)(groups < 148 * 16 * 256 ? ceil_div(groups, 256) : 148 * 16);
  if (groups < (int64_t)0xffffffffll - 148 * 16 * 256) {
    GRS_DTYPE_SWITCH(T, dtype,
        bias_gelu_kernel<T, uint32_t><<<grid, 256, 0, grs::counted((cudaStream_t)stream)>>>(
            (T*)y, rows, cols, stride, bias, apply_gelu))
  } else {
    GRS_DTYPE_SWITCH(T, dtype,
        bias_gelu_kernel<T, int64_t><<<grid, 256, 0, grs::counted((cudaStream_t)stream)>>>(
            (T*)y, rows, cols, stride, bias, apply_gelu))
  }
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_embed_initial(int dtype, const int64_t* types, int64_t rows, int width,
                                 const float* gate_emb, const float* marker, void* states,
                                 int64_t stride, uint8_t* live, void* stream) {
  if (rows <= 0) return GRS_OK;
  GRS_DTYPE_SWITCH(T, dtype, embed_initial_kernel<T><<<ceil_div(rows, ROW_WARPS), ROW_WARPS * 32, 0,
                                                       grs::counted((cudaStream_t)stream)>>>(
      types, rows, width, gate_emb, marker, (T*)states, stride, live))
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_graph_aggregate(int dtype, const void* fb, int64_t fb_stride, const float* rel,
                                   const int32_t* in_node, const int32_t* in_port,
                                   const int32_t* out_node, const int32_t* out_port, int64_t rows,
                                   int slots, int port_slots, int width, void* agg,
                                   int64_t agg_stride, void* stream) {
  if (rows <= 0) return GRS_OK;
  if (slots <= 0 || port_slots < slots) return GRS_ERR_SHAPE;
  const int grid = ceil_div(rows, ROW_WARPS);
  const int esize = dtype == GRS_DTYPE_F32 ? 4 : 2;
  const int vpl = width / 32;
  const int64_t vbytes = std::min<int64_t>(16, (int64_t)vpl * esize);
  const bool vec = width % 32 == 0 && vpl >= 2 && vpl <= 16 && vpl_for(width) == vpl &&
                   reinterpret_cast<uintptr_t>(fb) % vbytes == 0 &&
                   (fb_stride * esize) % vbytes == 0 && (width * esize) % vbytes == 0 &&
                   reinterpret_cast<uintptr_t>(agg) % vbytes == 0 &&
                   (agg_stride * esize) % vbytes == 0 && reinterpret_cast<uintptr_t>(rel) % 16 == 0 &&
                   ((reinterpret_cast<uintptr_t>(in_node) | reinterpret_cast<uintptr_t>(in_port) |
                     reinterpret_cast<uintptr_t>(out_node) | reinterpret_cast<uintptr_t>(out_port)) &
                    15) == 0;
  if (vec) {
    const int vgrid = ceil_div(rows, AGG_ROWS);
    const bool packed = fb_stride == 2 * width && agg_stride == 2 * width;
#define GRS_AGG_LAUNCH(PACKED)                                                                   \
    GRS_DTYPE_SWITCH(T, dtype, GRS_VPL_SWITCH(V, width,                                         \
        graph_aggregate_vec_kernel<T, V, PACKED><<<vgrid, ROW_WARPS * 32, 0,                    \
                                                   grs::counted((cudaStream_t)stream)>>>(       \
            (const T*)fb, fb_stride, rel, in_node, in_port, out_node, out_port, rows, slots,   \
            port_slots, (T*)agg, agg_stride)))
    if (packed) {
      GRS_AGG_LAUNCH(true)
    } else {
      GRS_AGG_LAUNCH(false)
    }
#undef GRS_AGG_LAUNCH
  } else {
    GRS_DTYPE_SWITCH(T, dtype, GRS_VPL_SWITCH(V, width,
        graph_aggregate_kernel<T, V><<<grid, ROW_WARPS * 32, 0, grs::counted((cudaStream_t)stream)>>>(
            (const T*)fb, fb_stride, rel, in_node, in_port, out_node, out_port, rows, slots,
            port_slots, width, (T*)agg, agg_stride)))
  }
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_action_inputs(int dtype, const void* states, int64_t state_stride, int slots,
                                 const int64_t* xfer_ids, const int64_t* source_ids,
                                 const int64_t* source_slots, int pattern, int width,
                                 const float* xfer_emb, const float* source_reps, void* bound,
                                 void* ctx_in, uint8_t* source_mask, uint8_t* active, int batch,
                                 void* stream) {
  if (batch <= 0) return GRS_OK;
  if (pattern > 32) return GRS_ERR_SHAPE;
  GRS_DTYPE_SWITCH(T, dtype, action_inputs_kernel<T><<<batch, 128, 0, grs::counted((cudaStream_t)stream)>>>(
      (const T*)states, state_stride, slots, xfer_ids, source_ids, source_slots, pattern, width,
      xfer_emb, source_reps, (T*)bound, (T*)ctx_in, source_mask, active, batch))
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_position_token(int dtype, const void* raw, const float* position,
                                  const int32_t* lengths, const uint8_t* active, void* token,
                                  int batch, int width, void* stream) {
  if (batch <= 0) return GRS_OK;
  const int64_t n = (int64_t)batch * width;
  GRS_DTYPE_SWITCH(T, dtype, position_token_kernel<T><<<ceil_div(n, 256), 256, 0, grs::counted((cudaStream_t)stream)>>>(
      (const T*)raw, position, lengths, active, (T*)token, batch, width))
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_update_live_hidden(int dtype, const void* qxa, int64_t qxa_stride,
                                      const void* keys, const void* vw, const void* cvec,
                                      const uint8_t* source_mask, int pattern, int64_t rows,
                                      int slots, int width, void* hidden, int64_t hidden_stride,
                                      float* affinity, void* stream) {
  if (rows <= 0) return GRS_OK;
  if (pattern <= 0 || pattern > 8 || slots <= 0 || rows % slots) return GRS_ERR_SHAPE;
  const int vq = vpl_for(width), vh = vpl_for(2 * width);
  if (vq < 0 || vh < 0 || width % vq || (2 * width) % vh) return GRS_ERR_SHAPE;
  // vector accesses: every row start aligned to the per-lane chunk (<= 16 B)
  const int esize = dtype == GRS_DTYPE_F32 ? 4 : 2;
  const int64_t aq = std::min(16, vq * esize), ah = std::min(16, vh * esize);
  if (((uintptr_t)qxa % aq) || ((qxa_stride * esize) % aq) || ((width * esize) % ah) ||
      ((uintptr_t)hidden % ah) || ((hidden_stride * esize) % ah))
    return GRS_ERR_SHAPE;
  const size_t smem = (size_t)(3 * pattern + 2) * width * sizeof(float);
  if (smem > 160 * 1024) return GRS_ERR_SHAPE;
  const dim3 grid(ceil_div(slots, ULH_ROWS), (unsigned)(rows / slots));
  const int interleave = width == 32 * vq && 2 * width == 32 * vh && vq % 4 == 0 && vh % 4 == 0;
#define GRS_ULH(VQ, VH)                                                                        \
  if (vq == VQ && vh == VH) {                                                                  \
    GRS_DTYPE_SWITCH(T, dtype,                                                                 \
        if (smem > 48 * 1024) cudaFuncSetAttribute(update_live_hidden_kernel<T, VQ, VH>,      \
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);     \
        update_live_hidden_kernel<T, VQ, VH><<<grid, ROW_WARPS * 32, smem,                     \
                                               grs::counted((cudaStream_t)stream)>>>(          \
        (const T*)qxa, qxa_stride, (const T*)keys, (const T*)vw, (const T*)cvec, source_mask,  \
        pattern, slots, width, (T*)hidden, hidden_stride, affinity, interleave))                \
    GRS_CUDA_CHECK_LAUNCH();                                                                   \
    return GRS_OK;                                                                             \
  }
  GRS_ULH(1, 2) GRS_ULH(2, 4) GRS_ULH(4, 8) GRS_ULH(8, 16) GRS_ULH(16, 32) GRS_ULH(1, 1)
  GRS_ULH(2, 2) GRS_ULH(4, 4) GRS_ULH(8, 8) GRS_ULH(16, 16)
#undef GRS_ULH
  return GRS_ERR_SHAPE;
}

extern "C" int grs_destination_hidden(int dtype, const void* r, const float* type_table,
                                      const float* pos_table, const int64_t* dest_slots,
                                      const int64_t* dest_types, const uint8_t* active,
                                      int pattern, int batch, int hidden_width, void* hidden,
                                      void* stream) {
  const int64_t n = (int64_t)batch * pattern * hidden_width;
  if (n <= 0) return GRS_OK;
  GRS_DTYPE_SWITCH(T, dtype, destination_hidden_kernel<T><<<ceil_div(n, 256), 256, 0, grs::counted((cudaStream_t)stream)>>>(
      (const T*)r, type_table, pos_table, dest_slots, dest_types, active, pattern, batch,
      hidden_width, (T*)hidden))
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_apply_slots(int dtype, void* states, int64_t state_stride, uint8_t* live,
                               int64_t* types, int slots, const int64_t* source_slots,
                               const uint8_t* source_mask, int spattern, const int64_t* dest_slots,
                               const int64_t* dest_types, const uint8_t* active, int dpattern,
                               const void* created, int width, int batch, void* stream) {
  if (batch <= 0) return GRS_OK;
  GRS_DTYPE_SWITCH(T, dtype, apply_slots_kernel<T><<<batch, 128, 0, grs::counted((cudaStream_t)stream)>>>(
      (T*)states, state_stride, live, types, slots, source_slots, source_mask, spattern,
      dest_slots, dest_types, active, dpattern, (const T*)created, width, batch))
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_match_logits(int dtype, const void* acc, int64_t acc_stride,
                                const float* source_bias, const int64_t* first_types,
                                const uint8_t* live, const int64_t* types, int64_t rows,
                                int num_sources, float inv_sqrt_r, float* logits,
                                uint8_t* eligible, void* stream) {
  const int64_t n = rows * num_sources;
  if (n <= 0) return GRS_OK;
  GRS_DTYPE_SWITCH(T, dtype, match_logits_kernel<T><<<ceil_div(n, 256), 256, 0, grs::counted((cudaStream_t)stream)>>>(
      (const T*)acc, acc_stride, source_bias, first_types, live, types, rows, num_sources,
      inv_sqrt_r, logits, eligible))
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_gather_beams(const void* in, void* out, const int64_t* index, int64_t rows,
                                int64_t in_bytes, int64_t out_bytes, int fill_byte,
                                void* stream) {
  if (rows <= 0) return GRS_OK;
  if (in_bytes < 0 || out_bytes < 0) return GRS_ERR_SHAPE;
  gather_beams_kernel<<<(unsigned)rows, 256, 0, grs::counted((cudaStream_t)stream)>>>(
      (const char*)in, (char*)out, index, rows, in_bytes, out_bytes, fill_byte);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_edges_to_ports(const int64_t* eb, const int64_t* es, const int64_t* ed,
                                  const int64_t* er, int64_t edges, int slots, int32_t* out_node,
                                  int32_t* out_port, int32_t* in_node, int32_t* in_port,
                                  void* stream) {
  if (edges <= 0) return GRS_OK;
  edges_to_ports_kernel<<<ceil_div(edges, 256), 256, 0, grs::counted((cudaStream_t)stream)>>>(
      eb, es, ed, er, edges, slots, out_node, out_port, in_node, in_port);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}
