// bf16 GEMMs with fused row epilogues on the 5th-generation tensor cores:
//   out[M, N] = epilogue(A[M, K] . B[N, K]^T)
// A is row-major with row stride lda, B is K-major (a PyTorch Linear weight
// [out, in]), fp32 accumulation in tensor memory.  These are every bf16
// projection of the paged action model (paged_model.py:36-94, 213-241,
// 338-436, 513-604; model.py:26-53, 375-389), each with the elementwise work
// that follows it in the reference folded into the epilogue so the [M, N]
// product is written once:
//
//   STORE      (+ bias) (+ residual) (GELU) (dead rows zeroed) -> bf16
//   LAYERNORM  N = 256: LayerNorm(residual + row_scale * (acc + bias)), rows
//              that keep their input (where masks) or are zeroed (zero_row)
//   LOGITS     N = 32: match logits (acc * scale + source bias) masked to the
//              eligible (slot, source) pairs, fp32 logits + eligibility
//
// Persistent and warp-specialised, one CTA per SM walking 128 x BN output
// tiles (consecutive tiles share their A rows): warp 0 (one thread) streams
// 64-wide K slices of A and B with TMA into a ring of shared-memory stages
// (128-byte swizzle); warp 1 (one thread) issues tcgen05.mma into one of two
// BN-column fp32 accumulators in TMEM and commits each stage back to the
// producer and each finished tile to the epilogue; the epilogue warps drain
// the other accumulator meanwhile (warp w reads TMEM lanes 32 (w % 4) and 64
// columns ((w - 2) / 4) of the tile), apply the epilogue, stage the bf16
// block in shared memory with the 128-byte swizzle and write it with a TMA
// store.  Every wait is bounded; a wait that gives up reports GRS_ERR_TIMEOUT.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "grs_common.cuh"
#include "sm100.cuh"

namespace grs {

constexpr int GT_BM = 128, GT_BK = 64, GT_ACC = 2;
constexpr int GT_A_BYTES = GT_BM * GT_BK * 2;                 // 16 KB
constexpr int GT_OUT_BYTES = 32 * 128;                        // one warp's 32 x 64 bf16 block

// Epilogue modes
constexpr int GT_EPI_STORE = 0, GT_EPI_LAYERNORM = 1, GT_EPI_LOGITS = 2;

// Tile geometry for a tile width BN (the MMA's N)
template <int BN>
struct GtShape {
  static constexpr int kB = BN * GT_BK * 2;                   // B stage bytes
  static constexpr int kStage = GT_A_BYTES + kB;
  static constexpr int kStages = BN == 256 ? 3 : BN == 128 ? 4 : 6;
  static constexpr int kEpiWarps = BN >= 64 ? 4 * (BN / 64) : 4;
  static constexpr int kThreads = (2 + kEpiWarps) * 32;
  // BN < 64 is the logits epilogue: each warp stages its 32 rows of <= 32
  // fp32 logits and <= 32 eligibility bytes
  static constexpr int kStaging = BN >= 64 ? kEpiWarps * GT_OUT_BYTES : kEpiWarps * 32 * 32 * 5;
  static constexpr int kSmem = kStages * kStage + kStaging + 1024;   // + alignment slack
};

struct GemmEpilogue {
  const float* bias;            // [N] or null
  int gelu;
  __nv_bfloat16* out;
  int64_t ldo;
  int32_t* status;
  const __nv_bfloat16* residual;   // [M, N] (STORE: added; LAYERNORM: the input) or null
  int64_t ldr;
  const float* row_scale;       // LAYERNORM: scales (acc + bias) per row, or null
  const float* gamma;
  const float* beta;
  const uint8_t* zero_row;      // rows whose output is zero, or null
  const uint8_t* where_row;     // LAYERNORM: rows with 0 keep the residual
  const uint8_t* where_beam;    // LAYERNORM: beams (row / rows_per_beam) with 0 keep it
  const int32_t* where_len;     // LAYERNORM: beams with length <= 0 keep it
  int rows_per_beam;
  float eps;
  // LOGITS
  float* logits;
  uint8_t* eligible;
  const int64_t* first_types;
  const uint8_t* live;
  const int64_t* types;
  int num_sources;
  float logit_scale;
};

// named barrier of the epilogue warps that share one TMEM lane quarter
// (`groups` warps of 64 columns each)
__device__ __forceinline__ void quarter_sync(int quarter, int groups = 4) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(1 + quarter), "r"(32 * groups) : "memory");
}

// erf-based GELU on fp32 pairs: Abramowitz & Stegun 7.1.28 for erfc (the
// same form as the row kernels' GELU), packed fp32x2 multiply-adds.
__device__ __forceinline__ float2 gelu_pair(float2 x) {
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

__device__ __forceinline__ void add_bias32(float v[32], const float* bias) {
  const float4* b4 = reinterpret_cast<const float4*>(bias);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 bb = __ldg(b4 + j);
    v[4 * j] += bb.x;
    v[4 * j + 1] += bb.y;
    v[4 * j + 2] += bb.z;
    v[4 * j + 3] += bb.w;
  }
}

// v[0..31] += 32 consecutive bf16 of a row (64 bytes, 16-byte aligned)
__device__ __forceinline__ void add_row32(float v[32], const __nv_bfloat16* src) {
  const uint4* x4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 w = x4[j];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __bfloat1622float2(h[k]);
      v[8 * j + 2 * k] += f.x;
      v[8 * j + 2 * k + 1] += f.y;
    }
  }
}

// chunk c (32 columns = four 16-byte pieces) of row `lane` of a warp's
// 32 x 64 bf16 staging block, placed by the 128-byte swizzle of the output
// tensor map (16-byte piece index ^ row % 8)
__device__ __forceinline__ void stage_row_chunks(uint8_t* stage, int lane, int c,
                                                 const uint32_t packed[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int chunk = c * 4 + j;
    *reinterpret_cast<uint4*>(stage + lane * 128 + ((chunk ^ (lane & 7)) << 4)) =
        make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
  }
}

// v[0..31] += chunk c (32 columns) of row `lane` of a warp's staging block
// (the residual, landed there by a TMA load in the output's swizzled layout)
__device__ __forceinline__ void add_staged32(float v[32], const uint8_t* stage, int lane, int c) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int chunk = c * 4 + j;
    const uint4 w = *reinterpret_cast<const uint4*>(stage + lane * 128 + ((chunk ^ (lane & 7)) << 4));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __bfloat1622float2(h[k]);
      v[8 * j + 2 * k] += f.x;
      v[8 * j + 2 * k + 1] += f.y;
    }
  }
}

// 64 consecutive bf16 of a row (128 bytes, 16-byte aligned) into registers,
// or zeros when the row is past the end
__device__ __forceinline__ void load_row64(const __nv_bfloat16* src, bool in, uint4 r[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    r[j] = in ? *reinterpret_cast<const uint4*>(src + 8 * j) : make_uint4(0, 0, 0, 0);
}

// v[0..31] += the 32 bf16 held in r[0..3]
__device__ __forceinline__ void add_regs32(float v[32], const uint4 r[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r[j]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __bfloat1622float2(h[k]);
      v[8 * j + 2 * k] += f.x;
      v[8 * j + 2 * k + 1] += f.y;
    }
  }
}

// exact mean and centred sum of squares of 64 values
__device__ __forceinline__ void stats64(const float v[64], float& mean, float& m2) {
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int j = 0; j < 64; j += 2) {
    s0 += v[j];
    s1 += v[j + 1];
  }
  mean = (s0 + s1) * (1.f / 64.f);
  float q0 = 0.f, q1 = 0.f;
#pragma unroll
  for (int j = 0; j < 64; j += 2) {
    const float d0 = v[j] - mean, d1 = v[j + 1] - mean;
    q0 = fmaf(d0, d0, q0);
    q1 = fmaf(d1, d1, q1);
  }
  m2 = q0 + q1;
}

__device__ __forceinline__ void pack_bf16x32(const float v[32], uint32_t packed[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
    packed[j] = *reinterpret_cast<uint32_t*>(&h);
  }
}

template <int BN, int MODE>
__global__ void __launch_bounds__(GtShape<BN>::kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
               const __grid_constant__ CUtensorMap tm_out, const __grid_constant__ CUtensorMap tm_res,
               int M, int N, int K, GemmEpilogue e) {
  using namespace sm100;
  using S = GtShape<BN>;
  extern __shared__ uint8_t gt_smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[S::kStages], empty_bar[S::kStages];
  // per epilogue warp: its residual block landed in its staging block
  __shared__ __align__(8) uint64_t res_bar[S::kEpiWarps];
  __shared__ __align__(8) uint64_t tmem_full[GT_ACC], tmem_empty[GT_ACC];
  __shared__ __align__(8) uint64_t drain_bar;   // completes when every issued MMA is done
  __shared__ uint32_t tmem_slot;
  __shared__ int failed, drain_failed;
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(gt_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k_iters = K / GT_BK;
  const int n_tiles = N / BN;
  const int tiles = ((M + GT_BM - 1) / GT_BM) * n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < GT_ACC; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], S::kEpiWarps);
    }
    mbar_init(&drain_bar, 1);
    for (int w = 0; w < S::kEpiWarps; ++w) mbar_init(&res_bar[w], 1);
    failed = 0;
    drain_failed = 0;
    mbar_init_fence();
  }
  if (warp == 0) tmem_alloc(&tmem_slot, GT_ACC * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer: the ring runs across tiles
      int g = 0;
      int armed[S::kStages] = {};   // phases armed per stage
      for (int t = blockIdx.x; t < tiles && !failed; t += gridDim.x) {
        const int m0 = (t / n_tiles) * GT_BM, n0 = (t % n_tiles) * BN;
        for (int it = 0; it < k_iters; ++it, ++g) {
          const int s = g % S::kStages, r = g / S::kStages;
          if (r > 0 && !mbar_wait(&empty_bar[s], (r - 1) & 1)) {
            failed = 1;
            break;
          }
          uint8_t* a = smem + s * S::kStage;
          mbar_arrive_expect_tx(&full_bar[s], S::kStage);
          tma_load_2d(a, &tm_a, it * GT_BK, m0, &full_bar[s]);
          tma_load_2d(a + GT_A_BYTES, &tm_b, it * GT_BK, n0, &full_bar[s]);
          armed[s] = r + 1;
        }
      }
      // every load in flight lands before the CTA exits: the last armed phase
      // of each stage (long completed when the MMA thread consumed it)
      for (int s = 0; s < S::kStages; ++s)
        if (armed[s] > 0 && !mbar_wait(&full_bar[s], (armed[s] - 1) & 1)) drain_failed = 1;
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      constexpr uint32_t idesc = idesc_bf16_f32(GT_BM, BN);
      int g = 0, i = 0;
      for (int t = blockIdx.x; t < tiles && !failed; t += gridDim.x, ++i) {
        const int b = i & 1, u = i >> 1;
        if (u > 0 && !mbar_wait(&tmem_empty[b], (u - 1) & 1)) {
          failed = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        for (int it = 0; it < k_iters; ++it, ++g) {
          const int s = g % S::kStages, r = g / S::kStages;
          if (!mbar_wait(&full_bar[s], r & 1)) {
            failed = 1;
            break;
          }
          tc_fence_after();
          const uint8_t* a = smem + s * S::kStage;
          const uint64_t ad = smem_desc_k128(a), bd = smem_desc_k128(a + GT_A_BYTES);
#pragma unroll
          for (int kk = 0; kk < GT_BK / 16; ++kk)  // 16 bf16 = 32 bytes = 2 descriptor units
            mma_bf16(acc, ad + 2 * kk, bd + 2 * kk, idesc, it > 0 || kk > 0);
          mma_commit(&empty_bar[s]);
        }
        mma_commit(&tmem_full[b]);
      }
      // no MMA may still write TMEM when it is freed, also after a wait gave up
      mma_commit(&drain_bar);
      if (!mbar_wait(&drain_bar, 0)) drain_failed = 1;
    }
  } else if constexpr (MODE == GT_EPI_STORE) {
    // TMEM -> registers -> bias, residual, GELU, mask -> bf16 -> smem -> TMA store
    const int quarter = warp & 3, cgroup = (warp - 2) >> 2;   // 64 columns per warp
    uint8_t* stage = smem + S::kStages * S::kStage + (warp - 2) * GT_OUT_BYTES;
    uint64_t* rbar = &res_bar[warp - 2];
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int m0 = (t / n_tiles) * GT_BM, n0 = (t % n_tiles) * BN;
      const int b = i & 1, u = i >> 1;
      const int row = m0 + quarter * 32 + lane;
      const bool in = row < M;
      const bool zero = in && e.zero_row != nullptr && e.zero_row[row] == 0;
      // the warp's residual block goes into its staging block (once the
      // previous output block has left it) while the MMAs run; rows past
      // the end read as zeros
      if (lane == 0) {
        tma_store_wait_read();
        if (e.residual) {
          mbar_arrive_expect_tx(rbar, GT_OUT_BYTES);
          tma_load_2d(stage, &tm_res, n0 + cgroup * 64, m0 + quarter * 32, rbar);
        }
      }
      __syncwarp();
      if (!mbar_wait_warp(&tmem_full[b], u & 1) ||
          (e.residual && !mbar_wait_warp(rbar, i & 1))) {
        failed = 1;
        // a residual load still in flight lands before the warp leaves
        if (lane == 0 && e.residual) mbar_wait(rbar, i & 1);
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        const int col = cgroup * 64 + c * 32;
        float v[32];
        tmem_load32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * BN + col), v);
        if (e.bias) add_bias32(v, e.bias + n0 + col);
        if (e.residual) add_staged32(v, stage, lane, c);
        if (e.gelu) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float2 p = gelu_pair(make_float2(v[2 * j], v[2 * j + 1]));
            v[2 * j] = p.x;
            v[2 * j + 1] = p.y;
          }
        }
        if (zero) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.f;
        }
        uint32_t packed[16];
        pack_bf16x32(v, packed);
        stage_row_chunks(stage, lane, c, packed);
      }
      tc_fence_before();
      fence_async_shared();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tmem_empty[b]);          // this warp is done with accumulator b
        tma_store_2d(&tm_out, stage, n0 + cgroup * 64, m0 + quarter * 32);
      }
    }
    if (lane == 0) tma_store_wait_all();
  } else if constexpr (MODE == GT_EPI_LAYERNORM) {
    // each row's BN columns are spread over the BN / 64 warps of its lane
    // quarter; per-warp (mean, centred sum of squares) pairs meet in shared
    // memory and merge exactly, so one pass over the accumulator gives the
    // statistics and a second writes the row
    static_assert(BN == 256 || BN == 128, "the LayerNorm epilogue normalises whole rows");
    constexpr int G = BN / 64;
    __shared__ float ln_part[4][4][32], ln_m2[4][4][32];
    const int quarter = warp & 3, cgroup = (warp - 2) >> 2;
    uint8_t* stage = smem + S::kStages * S::kStage + (warp - 2) * GT_OUT_BYTES;
    uint64_t* rbar = &res_bar[warp - 2];
    int i = 0, res_issued = 0, res_landed = 0;   // residual loads of this warp
    bool gave_up = false;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int m0 = t * GT_BM;                                 // N == BN: one tile per row block
      const int b = i & 1, u = i >> 1;
      // after a wait gave up, the warp still runs every named barrier so the
      // other warps of its quarter are not left waiting
      const int row = m0 + quarter * 32 + lane;
      const bool in = row < M;
      // the warp's residual block goes into its staging block (once the
      // previous output block has left it) and the row's scale and masks are
      // read before the wait: their latency hides behind the tile's MMAs
      const bool res_here = e.residual && !gave_up;
      if (lane == 0) {
        tma_store_wait_read();
        if (res_here) {
          mbar_arrive_expect_tx(rbar, GT_OUT_BYTES);
          tma_load_2d(stage, &tm_res, cgroup * 64, m0 + quarter * 32, rbar);
        }
      }
      res_issued += res_here ? 1 : 0;
      __syncwarp();
      const int64_t beam = in ? row / e.rows_per_beam : 0;
      const float sc = (in && e.row_scale) ? e.row_scale[row] : 1.f;
      bool zc = true, wc = true;
      if (in) {
        if (e.zero_row) zc = e.zero_row[row] != 0;
        if (e.where_row) wc = wc && e.where_row[row] != 0;
        if (e.where_beam) wc = wc && e.where_beam[beam] != 0;
        if (e.where_len) wc = wc && e.where_len[beam] > 0;
      }
      if (res_here) {
        if (mbar_wait_warp(rbar, (res_issued - 1) & 1)) {
          ++res_landed;
        } else {
          gave_up = true;
          failed = 1;
        }
      }
      if (!gave_up && !mbar_wait_warp(&tmem_full[b], u & 1)) {
        gave_up = true;
        failed = 1;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * BN);
      // v = residual + row_scale * (acc + bias) for one 32-column chunk
      const auto load_row = [&](int c, float v[32]) {
        const int col = cgroup * 64 + c * 32;
        tmem_load32(taddr + (uint32_t)col, v);
        add_bias32(v, e.bias + col);
        if (sc != 1.f) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] *= sc;
        }
        if (e.residual) add_staged32(v, stage, lane, c);
      };
      // this thread's 64 columns: exact mean and centred sum of squares of
      // each 32-column chunk, merged (Chan, Golub & LeVeque's pairwise update)
      float mean_t = 0.f, m2_t = 0.f;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float v[32];
        load_row(c, v);
        float mc = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) mc += v[j];
        mc *= (1.f / 32.f);
        float m2c = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float d = v[j] - mc;
          m2c += d * d;
        }
        if (c == 0) {
          mean_t = mc;
          m2_t = m2c;
        } else {                       // two halves of 32: n_a n_b / n = 16
          const float delta = mc - mean_t;
          mean_t += 0.5f * delta;
          m2_t += m2c + 16.f * delta * delta;
        }
      }
      ln_part[quarter][cgroup][lane] = mean_t;
      ln_m2[quarter][cgroup][lane] = m2_t;
      quarter_sync(quarter, G);
      // the row's 64-column groups, merged pairwise the same way
      const float* pm = &ln_part[quarter][0][lane];
      const float* p2 = &ln_m2[quarter][0][lane];
      const float d01 = pm[32] - pm[0];
      float mean = pm[0] + 0.5f * d01;
      float m2 = p2[0] + p2[32] + 32.f * d01 * d01;
      if constexpr (G == 4) {
        const float d23 = pm[96] - pm[64];
        const float mean23 = pm[64] + 0.5f * d23;
        const float m223 = p2[64] + p2[96] + 32.f * d23 * d23;
        const float dd = mean23 - mean;
        m2 += m223 + 64.f * dd * dd;
        mean += 0.5f * dd;
      }
      const float var = m2 * (1.f / BN);
      quarter_sync(quarter, G);
      const float rstd = rsqrtf(var + e.eps);
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        const int col = cgroup * 64 + c * 32;
        // the accumulator read (tcgen05.ld, a warp-collective instruction) is
        // made by every lane; the per-row masks only select what is written
        float r[32];
        load_row(c, r);
        if (!zc) {
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = 0.f;
        } else if (!wc) {             // the row keeps its input
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = 0.f;
          if (e.residual) add_staged32(r, stage, lane, c);
        } else {
          const float4* g4 = reinterpret_cast<const float4*>(e.gamma + col);
          const float4* b4 = reinterpret_cast<const float4*>(e.beta + col);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 g = __ldg(g4 + j), bb = __ldg(b4 + j);
            r[4 * j] = (r[4 * j] - mean) * rstd * g.x + bb.x;
            r[4 * j + 1] = (r[4 * j + 1] - mean) * rstd * g.y + bb.y;
            r[4 * j + 2] = (r[4 * j + 2] - mean) * rstd * g.z + bb.z;
            r[4 * j + 3] = (r[4 * j + 3] - mean) * rstd * g.w + bb.w;
          }
        }
        uint32_t packed[16];
        pack_bf16x32(r, packed);
        stage_row_chunks(stage, lane, c, packed);
      }
      tc_fence_before();
      fence_async_shared();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tmem_empty[b]);
        tma_store_2d(&tm_out, stage, cgroup * 64, m0 + quarter * 32);
      }
    }
    // a residual load that was not seen to land lands before the warp leaves
    if (lane == 0 && res_issued > res_landed) mbar_wait(rbar, (res_issued - 1) & 1);
    if (lane == 0) tma_store_wait_all();
  } else {
    // LOGITS (BN == 32): one thread per row reads its 32 accumulator columns;
    // a warp's 32 rows of logits (and of eligibility bytes) are contiguous in
    // the outputs, so they are staged in shared memory row by row and written
    // with 16-byte stores across the warp
    static_assert(BN == 32, "the logits epilogue reads one 32-column accumulator");
    const int quarter = warp & 3;
    const int ns = e.num_sources;
    float* lstage = reinterpret_cast<float*>(smem + S::kStages * S::kStage) + (warp - 2) * 32 * 32;
    uint8_t* estage = smem + S::kStages * S::kStage + S::kEpiWarps * 32 * 32 * 4 +
                      (warp - 2) * 32 * 32;
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int m0 = t * GT_BM;
      const int b = i & 1, u = i >> 1;
      const int r0 = m0 + quarter * 32;             // this warp's first row
      const int row = r0 + lane;
      const bool alive = row < M && e.live[row] != 0;
      const int64_t type = row < M ? e.types[row] : -1;
      if (!mbar_wait_warp(&tmem_full[b], u & 1)) {
        failed = 1;
        break;
      }
      tc_fence_after();
      float v[32];
      tmem_load32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * BN), v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[b]);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j < ns) {
          const bool ok = alive && type == __ldg(e.first_types + j);
          lstage[lane * ns + j] = ok ? v[j] * e.logit_scale + __ldg(e.bias + j) : -1e4f;
          estage[lane * ns + j] = ok;
        }
      }
      __syncwarp();
      const int rows = min(32, M - r0);
      float* lo = e.logits + (int64_t)r0 * ns;
      uint8_t* el = e.eligible + (int64_t)r0 * ns;
      const int nf = rows * ns, nb = rows * ns;
      if (((reinterpret_cast<uintptr_t>(lo) | reinterpret_cast<uintptr_t>(el)) & 15) == 0) {
        for (int k = lane; k < nf / 4; k += 32)
          reinterpret_cast<float4*>(lo)[k] = reinterpret_cast<const float4*>(lstage)[k];
        for (int k = (nf / 4) * 4 + lane; k < nf; k += 32) lo[k] = lstage[k];
        for (int k = lane; k < nb / 16; k += 32)
          reinterpret_cast<uint4*>(el)[k] = reinterpret_cast<const uint4*>(estage)[k];
        for (int k = (nb / 16) * 16 + lane; k < nb; k += 32) el[k] = estage[k];
      } else {
        for (int k = lane; k < nf; k += 32) lo[k] = lstage[k];
        for (int k = lane; k < nb; k += 32) el[k] = estage[k];
      }
      __syncwarp();
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  // a drain that gave up leaves the columns allocated rather than free them
  // under a pending MMA; the status word reports the timeout either way
  if (warp == 0 && !drain_failed) {
    tc_fence_after();
    tmem_dealloc(tmem, GT_ACC * BN);
  }
  if (threadIdx.x == 0 && (failed || drain_failed)) set_status(e.status, GRS_ERR_TIMEOUT);
}

// ---------------------------------------------------------------------------
// B-stationary store GEMM for K = 256: C[M, N] = A[M, 256] B[N, 256]^T
// (+ bias), rows with zero_row == 0 zeroed.  The model's K = 256 projections
// (node queries, the graph layers' fb, the update's query) are HBM-bound:
// their 256 x 256 weight tile is 2/3 of what the streaming kernel pulls
// into shared memory per output tile.  Here each CTA keeps its weight tile
// (all four K slices, 128 KB) resident for every tile it computes - the grid
// is a multiple of N / 256, so a CTA's tiles all share one column block -
// and only A streams through a five-stage ring.  Eight epilogue warps (two
// per TMEM lane quarter, 128 columns each) store 32 x 32 blocks with TMA
// through one 2 KB staging block each (64-byte swizzle): shared memory goes
// to A stages, which bound this kernel, rather than to deeper staging.
// ---------------------------------------------------------------------------
constexpr int BS_STAGES = 5;
constexpr int BS_K = 256;
constexpr int BS_KI = BS_K / GT_BK;                        // 4 K slices
constexpr int BS_B_SLICE = 256 * GT_BK * 2;                // 32 KB: 256 weight rows x 64
constexpr int BS_EPI_WARPS = 8, BS_THREADS = (2 + BS_EPI_WARPS) * 32;
constexpr int BS_STAGING = GT_OUT_BYTES / 2;             // one 32 x 32 bf16 block per warp
constexpr int BS_SMEM = BS_KI * BS_B_SLICE + BS_STAGES * GT_A_BYTES +
                        BS_EPI_WARPS * BS_STAGING + 1024;   // + alignment slack

__global__ void __launch_bounds__(BS_THREADS, 1)
gemm_bstat_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                  const __grid_constant__ CUtensorMap tm_out, int M, int N, GemmEpilogue e) {
  using namespace sm100;
  extern __shared__ uint8_t bs_smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[BS_STAGES], empty_bar[BS_STAGES];
  __shared__ __align__(8) uint64_t b_bar;                 // the weight tile has landed
  __shared__ __align__(8) uint64_t tmem_full[GT_ACC], tmem_empty[GT_ACC];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int failed, drain_failed;
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(bs_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* bsm = smem;                                     // 4 x 32 KB weight slices
  uint8_t* ring = bsm + BS_KI * BS_B_SLICE;                // 5 x 16 KB A stages
  uint8_t* stg = ring + BS_STAGES * GT_A_BYTES;            // 8 x 2 KB output blocks
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = N / 256;
  const int tiles = ((M + GT_BM - 1) / GT_BM) * n_tiles;
  const int n0 = (blockIdx.x % n_tiles) * 256;            // gridDim.x % n_tiles == 0

  if (threadIdx.x == 0) {
    for (int s = 0; s < BS_STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < GT_ACC; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], BS_EPI_WARPS);
    }
    mbar_init(&b_bar, 1);
    mbar_init(&drain_bar, 1);
    failed = 0;
    drain_failed = 0;
    mbar_init_fence();
  }
  if (warp == 0) tmem_alloc(&tmem_slot, GT_ACC * 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer: the weight tile once, then A slices
      mbar_arrive_expect_tx(&b_bar, BS_KI * BS_B_SLICE);
      for (int k = 0; k < BS_KI; ++k)
        tma_load_2d(bsm + k * BS_B_SLICE, &tm_b, k * GT_BK, n0, &b_bar);
      int g = 0;
      int armed[BS_STAGES] = {};
      for (int t = blockIdx.x; t < tiles && !failed; t += gridDim.x) {
        const int m0 = (t / n_tiles) * GT_BM;
        for (int it = 0; it < BS_KI; ++it, ++g) {
          const int s = g % BS_STAGES, r = g / BS_STAGES;
          if (r > 0 && !mbar_wait(&empty_bar[s], (r - 1) & 1)) {
            failed = 1;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[s], GT_A_BYTES);
          tma_load_2d(ring + s * GT_A_BYTES, &tm_a, it * GT_BK, m0, &full_bar[s]);
          armed[s] = r + 1;
        }
      }
      // every load in flight lands before the CTA exits
      if (!mbar_wait(&b_bar, 0)) drain_failed = 1;
      for (int s = 0; s < BS_STAGES; ++s)
        if (armed[s] > 0 && !mbar_wait(&full_bar[s], (armed[s] - 1) & 1)) drain_failed = 1;
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      constexpr uint32_t idesc = idesc_bf16_f32(GT_BM, 256);
      if (!mbar_wait(&b_bar, 0)) failed = 1;
      tc_fence_after();
      int g = 0, i = 0;
      for (int t = blockIdx.x; t < tiles && !failed; t += gridDim.x, ++i) {
        const int b = i & 1, u = i >> 1;
        if (u > 0 && !mbar_wait(&tmem_empty[b], (u - 1) & 1)) {
          failed = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * 256);
        for (int it = 0; it < BS_KI; ++it, ++g) {
          const int s = g % BS_STAGES, r = g / BS_STAGES;
          if (!mbar_wait(&full_bar[s], r & 1)) {
            failed = 1;
            break;
          }
          tc_fence_after();
          const uint64_t ad = smem_desc_k128(ring + s * GT_A_BYTES);
          const uint64_t bd = smem_desc_k128(bsm + it * BS_B_SLICE);
#pragma unroll
          for (int kk = 0; kk < GT_BK / 16; ++kk)
            mma_bf16(acc, ad + 2 * kk, bd + 2 * kk, idesc, it > 0 || kk > 0);
          mma_commit(&empty_bar[s]);
        }
        mma_commit(&tmem_full[b]);
      }
      mma_commit(&drain_bar);
      if (!mbar_wait(&drain_bar, 0)) drain_failed = 1;
    }
  } else {
    // TMEM -> registers -> bias, mask -> bf16 -> smem -> TMA store; warp
    // (quarter, half) drains lanes 32 quarter.. and columns 128 half.. as
    // four 32 x 32 blocks through its 2 KB staging block (64-byte swizzle)
    const int ew = warp - 2, quarter = warp & 3, half = ew >> 2;
    uint8_t* stage = stg + ew * BS_STAGING;
    const int sw = (lane >> 1) & 3;                  // 64-byte swizzle of row `lane`
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int m0 = (t / n_tiles) * GT_BM;
      const int b = i & 1, u = i >> 1;
      const int row = m0 + quarter * 32 + lane;
      const bool zero = row < M && e.zero_row != nullptr && e.zero_row[row] == 0;
      if (!mbar_wait_warp(&tmem_full[b], u & 1)) {
        failed = 1;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        const int col0 = half * 128 + c * 32;
        uint8_t* buf = stage;
        if (lane == 0) tma_store_wait_read();        // the last block's store has left it
        __syncwarp();
        float v[32];
        tmem_load32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * 256 + col0), v);
        if (e.bias) add_bias32(v, e.bias + n0 + col0);
        if (zero) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.f;
        }
        uint32_t packed[16];
        pack_bf16x32(v, packed);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(buf + lane * 64 + ((j ^ sw) << 4)) =
              make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
        fence_async_shared();
        __syncwarp();
        if (lane == 0) tma_store_2d(&tm_out, buf, n0 + col0, m0 + quarter * 32);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[b]);  // this warp is done with accumulator b
    }
    if (lane == 0) tma_store_wait_all();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 0 && !drain_failed) {
    tc_fence_after();
    tmem_dealloc(tmem, GT_ACC * 256);
  }
  if (threadIdx.x == 0 && (failed || drain_failed)) set_status(e.status, GRS_ERR_TIMEOUT);
}

// ---- host --------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 gemm_encode_fn() {
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

// [rows, cols] bf16 row-major (row stride `ld` elements) in boxes of 64
// columns x box_rows rows with the 128-byte swizzle, or of 32 columns with
// the 64-byte swizzle; a small cache keyed by every encoded field.
bool gemm_map(CUtensorMap* out, const void* base, int64_t rows, int64_t cols, int64_t ld,
              int box_rows, int box_cols = 64) {
  struct Key { const void* base; int64_t rows, cols, ld; int box, box_cols; };
  constexpr int kCache = 64;
  static Key keys[kCache];
  static CUtensorMap maps[kCache];
  static int used = 0, next = 0;
  static std::mutex mu;
  Key k;
  std::memset(&k, 0, sizeof(k));
  k.base = base; k.rows = rows; k.cols = cols; k.ld = ld; k.box = box_rows; k.box_cols = box_cols;
  if (box_cols != 64 && box_cols != 32) return false;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (std::memcmp(&keys[i], &k, sizeof(Key)) == 0) {
      *out = maps[i];
      return true;
    }
  auto fn = gemm_encode_fn();
  if (!fn) return false;
  cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t gstr[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows}, estr[2] = {1, 1};
  CUtensorMap m;
  if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), gdim, gstr, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE,
         box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  keys[next] = k;
  maps[next] = m;
  next = (next + 1) % kCache;
  used = used < kCache ? used + 1 : kCache;
  *out = m;
  return true;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int BN, int MODE>
int launch_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N, int K,
                void* out, int64_t ldo, const GemmEpilogue& e, cudaStream_t stream) {
  using S = GtShape<BN>;
  if (M <= 0) return GRS_OK;
  if (N <= 0 || K <= 0 || K % GT_BK || N % BN || lda % 8 || ldb % 8 || lda < K || ldb < K)
    return GRS_ERR_SHAPE;
  if (!aligned16(a) || !aligned16(b) || !aligned16(e.bias)) return GRS_ERR_SHAPE;
  if (MODE != GT_EPI_LOGITS && (ldo % 8 || ldo < N || !aligned16(out))) return GRS_ERR_SHAPE;
  if (e.residual && (e.ldr % 8 || e.ldr < N || !aligned16(e.residual))) return GRS_ERR_SHAPE;
  CUtensorMap tm_a, tm_b, tm_out, tm_res;
  if (!gemm_map(&tm_a, a, M, K, lda, GT_BM) || !gemm_map(&tm_b, b, N, K, ldb, BN))
    return GRS_ERR_SHAPE;
  if (MODE != GT_EPI_LOGITS) {
    if (!gemm_map(&tm_out, out, M, N, ldo, 32)) return GRS_ERR_SHAPE;
  } else {
    std::memset(&tm_out, 0, sizeof(tm_out));
  }
  // the residual is loaded in the output's 32-row x 64-column blocks
  if (MODE != GT_EPI_LOGITS && e.residual) {
    if (!gemm_map(&tm_res, e.residual, M, N, e.ldr, 32)) return GRS_ERR_SHAPE;
  } else {
    std::memset(&tm_res, 0, sizeof(tm_res));
  }
  static bool attr[64] = {};
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(gemm_tc_kernel<BN, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         S::kSmem);
    attr[dev] = true;
  }
  if (dev < 64 && !sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int64_t tiles = (int64_t)((M + GT_BM - 1) / GT_BM) * (N / BN);
  const int grid = (int)std::min<int64_t>(tiles, dev < 64 && sms[dev] ? sms[dev] : 148);
  gemm_tc_kernel<BN, MODE><<<grid, S::kThreads, S::kSmem, counted(stream)>>>(
      tm_a, tm_b, tm_out, tm_res, M, N, K, e);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

GemmEpilogue store_epilogue(const float* bias, int gelu, void* out, int64_t ldo,
                            const void* residual, int64_t ldr, const uint8_t* zero_row,
                            int32_t* status) {
  GemmEpilogue e;
  std::memset(&e, 0, sizeof(e));
  e.bias = bias;
  e.gelu = gelu;
  e.out = static_cast<__nv_bfloat16*>(out);
  e.ldo = ldo;
  e.status = status;
  e.residual = static_cast<const __nv_bfloat16*>(residual);
  e.ldr = ldr;
  e.zero_row = zero_row;
  e.rows_per_beam = 1;
  return e;
}

// The B-stationary kernel for a K = 256 store GEMM (no residual, no GELU)
// with enough row blocks that one CTA per SM, a multiple of N / 256 of them,
// stays busy.  Returns -1 when the shape is not one it takes.
int launch_bstat(const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N, int K,
                 void* out, int64_t ldo, const GemmEpilogue& e, cudaStream_t stream) {
  if (K != BS_K || N % 256 || e.residual || e.gelu || M <= 0) return -1;
  if (lda % 8 || ldb % 8 || lda < K || ldb < K || ldo % 8 || ldo < N) return -1;
  if (!aligned16(a) || !aligned16(b) || !aligned16(e.bias) || !aligned16(out)) return -1;
  static bool attr[64] = {};
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int n_tiles = N / 256;
  const int64_t row_blocks = (M + GT_BM - 1) / GT_BM;
  const int sm_count = dev < 64 && sms[dev] ? sms[dev] : 148;
  const int grid = (sm_count / n_tiles) * n_tiles;
  if (grid == 0 || row_blocks * n_tiles < 4 * (int64_t)grid) return -1;
  CUtensorMap tm_a, tm_b, tm_out;
  if (!gemm_map(&tm_a, a, M, K, lda, GT_BM) || !gemm_map(&tm_b, b, N, K, ldb, 256) ||
      !gemm_map(&tm_out, out, M, N, ldo, 32, 32))
    return GRS_ERR_SHAPE;
  if (dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(gemm_bstat_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             BS_SMEM) != cudaSuccess)
      return GRS_ERR_CUDA;
    attr[dev] = true;
  }
  gemm_bstat_kernel<<<grid, BS_THREADS, BS_SMEM, counted(stream)>>>(tm_a, tm_b, tm_out, M, N, e);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

}  // namespace
}  // namespace grs

using namespace grs;

extern "C" int grs_gemm_bf16(const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N,
                             int K, const float* bias, int gelu, const void* residual,
                             int64_t ldr, const uint8_t* zero_row, void* out, int64_t ldo,
                             int32_t* status, void* stream) {
  const GemmEpilogue e = store_epilogue(bias, gelu, out, ldo, residual, ldr, zero_row, status);
  // short GEMMs (the per-beam token path: M = beams) are latency-bound and
  // fill few SMs with 256-column tiles; 128-column tiles give twice the CTAs,
  // each with half the operand bytes and MMAs
  const int64_t tiles256 = (int64_t)((M + GT_BM - 1) / GT_BM) * (N / 256);
  const int bstat = launch_bstat(a, lda, b, ldb, M, N, K, out, ldo, e, (cudaStream_t)stream);
  if (bstat >= 0) return bstat;
  if (N % 256 == 0 && tiles256 >= 64)
    return launch_gemm<256, GT_EPI_STORE>(a, lda, b, ldb, M, N, K, out, ldo, e,
                                          (cudaStream_t)stream);
  if (N % 128 == 0)
    return launch_gemm<128, GT_EPI_STORE>(a, lda, b, ldb, M, N, K, out, ldo, e,
                                          (cudaStream_t)stream);
  return GRS_ERR_SHAPE;
}

extern "C" int grs_gemm_bf16_epilogue(const void* a, int64_t lda, const void* b, int64_t ldb,
                                      int M, int N, int K, const float* bias, int gelu,
                                      void* out, int64_t ldo, int32_t* status, void* stream) {
  return grs_gemm_bf16(a, lda, b, ldb, M, N, K, bias, gelu, nullptr, 0, nullptr, out, ldo,
                       status, stream);
}

extern "C" int grs_gemm_bf16_layernorm_ex(const void* a, int64_t lda, const void* b, int64_t ldb,
                                          int M, int N, int K, const float* bias,
                                          const float* row_scale, const void* residual,
                                          int64_t ldr, const float* gamma, const float* beta,
                                          const uint8_t* zero_row, const uint8_t* where_row,
                                          const uint8_t* where_beam, const int32_t* where_len,
                                          int rows_per_beam, float eps, void* out, int64_t ldo,
                                          int32_t* status, void* stream) {
  if (bias == nullptr || residual == nullptr || gamma == nullptr || beta == nullptr ||
      !aligned16(gamma) || !aligned16(beta) || rows_per_beam <= 0)
    return GRS_ERR_SHAPE;
  GemmEpilogue e = store_epilogue(bias, 0, out, ldo, residual, ldr, zero_row, status);
  e.row_scale = row_scale;
  e.gamma = gamma;
  e.beta = beta;
  e.where_row = where_row;
  e.where_beam = where_beam;
  e.where_len = where_len;
  e.rows_per_beam = rows_per_beam;
  e.eps = eps;
  if (N == 256)
    return launch_gemm<256, GT_EPI_LAYERNORM>(a, lda, b, ldb, M, 256, K, out, ldo, e,
                                              (cudaStream_t)stream);
  if (N == 128)
    return launch_gemm<128, GT_EPI_LAYERNORM>(a, lda, b, ldb, M, 128, K, out, ldo, e,
                                              (cudaStream_t)stream);
  return GRS_ERR_SHAPE;
}

extern "C" int grs_gemm_bf16_layernorm(const void* a, int64_t lda, const void* b, int64_t ldb,
                                       int M, int K, const float* bias, const void* residual,
                                       int64_t ldr, const float* gamma, const float* beta,
                                       const uint8_t* zero_row, float eps, void* out,
                                       int64_t ldo, int32_t* status, void* stream) {
  return grs_gemm_bf16_layernorm_ex(a, lda, b, ldb, M, 256, K, bias, nullptr, residual, ldr, gamma,
                                    beta, zero_row, nullptr, nullptr, nullptr, 1, eps, out, ldo,
                                    status, stream);
}

extern "C" int grs_match_logits_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                     int M, int K, int num_sources, const float* bias,
                                     const int64_t* first_types, const uint8_t* live,
                                     const int64_t* types, float scale, float* logits,
                                     uint8_t* eligible, int32_t* status, void* stream) {
  if (num_sources <= 0 || num_sources > 32 || !bias || !first_types || !live || !types ||
      !logits || !eligible)
    return GRS_ERR_SHAPE;
  GemmEpilogue e = store_epilogue(bias, 0, nullptr, 0, nullptr, 0, nullptr, status);
  e.logits = logits;
  e.eligible = eligible;
  e.first_types = first_types;
  e.live = live;
  e.types = types;
  e.num_sources = num_sources;
  e.logit_scale = scale;
  return launch_gemm<32, GT_EPI_LOGITS>(x, ldx, w, ldw, M, 32, K, nullptr, 0, e,
                                        (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// Fused graph-layer MLP (model.py:26-53, InitialGraphLayer's update and norm):
//   out = LayerNorm(x + GELU([x | agg] . U0^T + b0) . U2^T + b2) * live
// with A = [x | agg] bf16 [M, 512], U0 [512, 512], U2 [256, 512] K-major.
// The [M, 512] GELU activation never leaves the SM: per 128-row tile the
// first GEMM runs as two 256-column halves into the two halves of TMEM, the
// epilogue warps drain each half (bias, GELU, bf16) into a 64 KB
// shared-memory tile written in the 128-byte-swizzled K-major layout a TMA
// load would produce, and that tile is the A operand of the second GEMM:
// its first K half is consumed before the epilogue writes the second half
// into the same 64 KB, so the operand ring keeps three stages in flight.
// The residual enters the second GEMM's accumulator on the tensor cores:
// its 64-column slices ride in the otherwise unused A halves of the second
// GEMM's first four ring stages and are multiplied by a 16 x 16 identity
// held in shared memory (exact: bf16 x 1.0, fp32 accumulate), so the
// epilogue never loads it.  The epilogue adds b2, normalises the 256-column
// row, zeroes dead rows and writes the result with TMA stores (staged in the
// hidden tile, free by then).  TMEM halves alternate roles from tile to tile
// so the next tile's first GEMM overlaps this tile's LayerNorm.
// ---------------------------------------------------------------------------
namespace grs {

constexpr int GM_STAGES = 3;
constexpr int GM_B_BYTES = 256 * GT_BK * 2;                  // 32 KB: 256 weight rows x 64
constexpr int GM_STAGE = GT_A_BYTES + GM_B_BYTES;            // 48 KB
constexpr int GM_H_BYTES = 4 * GT_A_BYTES;                   // 64 KB: 128 x 256 bf16, one K half
constexpr int GM_LN_BYTES = 2 * 4 * 4 * 32 * 4;              // LayerNorm partials: 4 KB
// B operand of the residual MMAs: 16 rows x 64 K bf16 in the 128-byte
// swizzled K-major layout, row n holding 1.0 at the K columns k with
// k % 16 == n, so each 16-column K chunk of it is the 16 x 16 identity
constexpr int GM_ID_BYTES = 16 * 128;
constexpr int GM_EPI_WARPS = 16, GM_THREADS = (2 + GM_EPI_WARPS) * 32;
constexpr int GM_CTRL = 1024;                                // barriers, flags
constexpr int GM_SMEM = GM_CTRL + GM_STAGES * GM_STAGE + GM_H_BYTES + GM_LN_BYTES + GM_ID_BYTES +
                        1024;                                // + alignment slack

struct GraphMlpArgs {
  const float* b0;                  // [512]
  const float* b2;                  // [256]
  const float* gamma;
  const float* beta;
  const uint8_t* zero_row;          // live rows (0 = dead: written as zeros), or null
  float eps;
  int32_t* status;
};

// named barrier of all 16 epilogue warps
__device__ __forceinline__ void epilogue_sync() {
  asm volatile("bar.sync 5, 512;\n" ::: "memory");
}

__global__ void __launch_bounds__(GM_THREADS, 1)
graph_mlp_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_u0,
                 const __grid_constant__ CUtensorMap tm_u2, const __grid_constant__ CUtensorMap tm_res,
                 const __grid_constant__ CUtensorMap tm_out, int M, GraphMlpArgs e) {
  using namespace sm100;
  extern __shared__ uint8_t gm_smem_raw[];
  // control block, then 1024-aligned ring and hidden tile
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(gm_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(base);               // [2]
  uint64_t* empty_bar = full_bar + GM_STAGES;                           // [2]
  uint64_t* p1a_full = empty_bar + GM_STAGES;   // first half of GEMM 1 done
  uint64_t* p1b_full = p1a_full + 1;            // second half of GEMM 1 done
  uint64_t* p2_full = p1b_full + 1;             // GEMM 2 done
  // per 64-column hidden slice c (written by the 4 epilogue warps of column
  // group c, read by GEMM 2's K slices c and c + 4):
  uint64_t* g2a_done = p2_full + 1;             // [4] GEMM 2 K slice c done (slice free)
  uint64_t* h0_done = g2a_done + 4;             // [4] first-half slice c written
  uint64_t* h1_done = h0_done + 4;              // [4] second-half slice c written
  uint64_t* out_done = h1_done + 4;             // GEMM 2 accumulator drained (16 warps)
  uint64_t* drain_bar = out_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  int* failed = reinterpret_cast<int*>(tmem_slot + 1);
  int* drain_failed = failed + 1;
  uint8_t* ring = base + GM_CTRL;
  uint8_t* hid = ring + GM_STAGES * GM_STAGE;                           // 4 slices of 16 KB
  float* ln_part = reinterpret_cast<float*>(hid + GM_H_BYTES);          // [4][4][32]
  float* ln_m2 = ln_part + 4 * 4 * 32;
  uint8_t* ident = hid + GM_H_BYTES + GM_LN_BYTES;                      // 1024-aligned
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (M + GT_BM - 1) / GT_BM;
  constexpr int KI = 512 / GT_BK;                                       // 8 K slices

  if (threadIdx.x < GM_ID_BYTES / 16) {
    // 16-byte piece p of row n holds the K columns of logical piece p ^ (n % 8)
    const int n = threadIdx.x >> 3, piece = (threadIdx.x & 7) ^ (n & 7);
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k0 = piece * 8 + 2 * j;
      w[j] = (((k0 & 15) == n) ? 0x3F80u : 0u) | (((k0 + 1) & 15) == n ? 0x3F800000u : 0u);
    }
    *reinterpret_cast<uint4*>(ident + threadIdx.x * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    fence_async_shared();                  // visible to the tensor cores
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < GM_STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(p1a_full, 1);
    mbar_init(p1b_full, 1);
    mbar_init(p2_full, 1);
    for (int c = 0; c < 4; ++c) {
      mbar_init(&g2a_done[c], 1);
      mbar_init(&h0_done[c], GM_EPI_WARPS / 4);
      mbar_init(&h1_done[c], GM_EPI_WARPS / 4);
    }
    mbar_init(out_done, GM_EPI_WARPS);
    mbar_init(drain_bar, 1);
    *failed = 0;
    *drain_failed = 0;
    mbar_init_fence();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer: per tile 8 (A, U0 rows 0-255) + 8 (A, U0 rows 256-511) +
                      // 8 U2 slices, the first four with a 64-column residual slice
      int g = 0;
      int armed[GM_STAGES] = {};
      for (int t = blockIdx.x; t < tiles && !*failed; t += gridDim.x) {
        const int m0 = t * GT_BM;
        for (int it = 0; it < 3 * KI && !*failed; ++it, ++g) {
          const int s = g % GM_STAGES, r = g / GM_STAGES;
          if (r > 0 && !mbar_wait(&empty_bar[s], (r - 1) & 1)) {
            *failed = 1;
            break;
          }
          uint8_t* st = ring + s * GM_STAGE;
          const int phase = it / KI, k = it % KI;
          if (phase < 2) {
            mbar_arrive_expect_tx(&full_bar[s], GM_STAGE);
            tma_load_2d(st, &tm_a, k * GT_BK, m0, &full_bar[s]);
            tma_load_2d(st + GT_A_BYTES, &tm_u0, k * GT_BK, phase * 256, &full_bar[s]);
          } else if (k < 4) {
            mbar_arrive_expect_tx(&full_bar[s], GM_STAGE);
            tma_load_2d(st, &tm_res, k * GT_BK, m0, &full_bar[s]);
            tma_load_2d(st + GT_A_BYTES, &tm_u2, k * GT_BK, 0, &full_bar[s]);
          } else {
            mbar_arrive_expect_tx(&full_bar[s], GM_B_BYTES);
            tma_load_2d(st + GT_A_BYTES, &tm_u2, k * GT_BK, 0, &full_bar[s]);
          }
          armed[s] = r + 1;
        }
      }
      for (int s = 0; s < GM_STAGES; ++s)
        if (armed[s] > 0 && !mbar_wait(&full_bar[s], (armed[s] - 1) & 1)) *drain_failed = 1;
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      constexpr uint32_t idesc = idesc_bf16_f32(GT_BM, 256);
      constexpr uint32_t idesc_res = idesc_bf16_f32(GT_BM, 16);
      const uint64_t id_desc = smem_desc_k128(ident);
      int g = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
        const uint32_t x_reg = tmem + (uint32_t)((i & 1) * 256);        // GEMM 1a and GEMM 2
        const uint32_t y_reg = tmem + (uint32_t)(((i + 1) & 1) * 256);  // GEMM 1b
        for (int phase = 0; phase < 3 && ok; ++phase) {
          // the accumulator must be free: the last tile's second GELU half
          // drained (all four slices) or its LayerNorm done
          if (phase == 0 && i > 0)
            for (int c = 0; c < 4 && ok; ++c) ok = mbar_wait(&h1_done[c], (i - 1) & 1);
          if (phase == 1 && i > 0) ok = mbar_wait(out_done, (i - 1) & 1);
          if (!ok) break;
          tc_fence_after();
          const uint32_t acc = phase == 1 ? y_reg : x_reg;
          for (int k = 0; k < KI; ++k, ++g) {
            if (phase == 2) {
              // GEMM 2's K slice k reads hidden slice k % 4 of half k / 4,
              // as soon as its four warps have written it
              if (!mbar_wait(k < KI / 2 ? &h0_done[k] : &h1_done[k - KI / 2], i & 1)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            const int s = g % GM_STAGES, r = g / GM_STAGES;
            if (!mbar_wait(&full_bar[s], r & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint8_t* st = ring + s * GM_STAGE;
            const uint64_t ad =
                smem_desc_k128(phase < 2 ? st : hid + (k % (KI / 2)) * GT_A_BYTES);
            const uint64_t bd = smem_desc_k128(st + GT_A_BYTES);
#pragma unroll
            for (int kk = 0; kk < GT_BK / 16; ++kk)
              mma_bf16(acc, ad + 2 * kk, bd + 2 * kk, idesc, k > 0 || kk > 0);
            if (phase == 2 && k < 4) {
              // residual columns 64k + 16kk.. += residual slice . identity
              const uint64_t rd = smem_desc_k128(st);
#pragma unroll
              for (int kk = 0; kk < GT_BK / 16; ++kk)
                mma_bf16(acc + (uint32_t)(k * GT_BK + kk * 16), rd + 2 * kk, id_desc + 2 * kk,
                         idesc_res, true);
            }
            mma_commit(&empty_bar[s]);
            // the first-half slice is consumed: its warps may write their
            // second-half slice over it once these MMAs are done
            if (phase == 2 && k < KI / 2) mma_commit(&g2a_done[k]);
          }
          if (!ok) break;
          mma_commit(phase == 0 ? p1a_full : phase == 1 ? p1b_full : p2_full);
        }
      }
      if (!ok) *failed = 1;
      mma_commit(drain_bar);
      if (!mbar_wait(drain_bar, 0)) *drain_failed = 1;
    }
  } else {
    // epilogue warps: warp w reads TMEM lanes 32 (w % 4), 64 columns from ((w - 2) / 4) * 64
    const int quarter = warp & 3, cgroup = (warp - 2) >> 2;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    int i = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int m0 = t * GT_BM;
      const int row = m0 + quarter * 32 + lane;
      const bool in = row < M;
      const uint32_t x_reg = tmem + (uint32_t)((i & 1) * 256);
      const uint32_t y_reg = tmem + (uint32_t)(((i + 1) & 1) * 256);
      // ---- GELU halves into the hidden tile (slices half * 4 + cgroup)
      if (lane == 0) tma_store_wait_read();    // last tile's output staging has left smem
      __syncwarp();
      for (int half = 0; half < 2; ++half) {
        if (ok && !mbar_wait_warp(half == 0 ? p1a_full : p1b_full, i & 1)) {
          ok = false;
          *failed = 1;
        }
        // the second half overwrites the first once GEMM 2 has consumed it
        if (half == 1 && ok && !mbar_wait_warp(&g2a_done[cgroup], i & 1)) {
          ok = false;
          *failed = 1;
        }
        tc_fence_after();
        const uint32_t src = (half == 0 ? x_reg : y_reg) + (uint32_t)(cgroup * 64);
        uint8_t* dst = hid + cgroup * GT_A_BYTES + quarter * 32 * 128;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          float v[32];
          tmem_load32(src + lane_base + c * 32, v);
          add_bias32(v, e.b0 + half * 256 + cgroup * 64 + c * 32);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float2 p = gelu_pair(make_float2(v[2 * j], v[2 * j + 1]));
            v[2 * j] = p.x;
            v[2 * j + 1] = p.y;
          }
          uint32_t packed[16];
          pack_bf16x32(v, packed);
          stage_row_chunks(dst, lane, c, packed);
        }
        fence_async_shared();                  // hidden tile visible to the tensor cores
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(half == 0 ? &h0_done[cgroup] : &h1_done[cgroup]);
      }
      // ---- GEMM 2 epilogue (the accumulator holds the residual already):
      // + b2, LayerNorm, dead rows, TMA store.  The live flag is read before
      // the wait, so its latency hides behind the second GEMM.
      const bool keep = !in || e.zero_row == nullptr || e.zero_row[row] != 0;
      if (ok && !mbar_wait_warp(p2_full, i & 1)) {
        ok = false;
        *failed = 1;
      }
      tc_fence_after();
      const uint32_t taddr = x_reg + lane_base + (uint32_t)(cgroup * 64);
      // v = acc + b2 for one 32-column chunk (the accumulator is read twice,
      // once for the statistics and once for the output)
      const auto load_row = [&](int c, float v[32]) {
        tmem_load32(taddr + c * 32, v);
        add_bias32(v, e.b2 + cgroup * 64 + c * 32);
      };
      float mean_t = 0.f, m2_t = 0.f;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float v[32];
        load_row(c, v);
        float mc = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) mc += v[j];
        mc *= (1.f / 32.f);
        float m2c = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float d = v[j] - mc;
          m2c = fmaf(d, d, m2c);
        }
        if (c == 0) {
          mean_t = mc;
          m2_t = m2c;
        } else {                       // two halves of 32: n_a n_b / n = 16
          const float delta = mc - mean_t;
          mean_t += 0.5f * delta;
          m2_t += m2c + 16.f * delta * delta;
        }
      }
      ln_part[(quarter * 4 + cgroup) * 32 + lane] = mean_t;
      ln_m2[(quarter * 4 + cgroup) * 32 + lane] = m2_t;
      quarter_sync(quarter);
      const float* pm = ln_part + quarter * 128 + lane;
      const float* p2 = ln_m2 + quarter * 128 + lane;
      const float d01 = pm[32] - pm[0], d23 = pm[96] - pm[64];
      const float mean01 = pm[0] + 0.5f * d01, mean23 = pm[64] + 0.5f * d23;
      const float m201 = p2[0] + p2[32] + 32.f * d01 * d01;
      const float m223 = p2[64] + p2[96] + 32.f * d23 * d23;
      const float dd = mean23 - mean01;
      const float mean = mean01 + 0.5f * dd;
      const float var = (m201 + m223 + 64.f * dd * dd) * (1.f / 256.f);
      const float rstd = rsqrtf(var + e.eps);
      uint8_t* stage = hid + cgroup * GT_A_BYTES + quarter * 32 * 128;   // this warp's block
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float v[32];
        load_row(c, v);
        const float4* g4 = reinterpret_cast<const float4*>(e.gamma + cgroup * 64 + c * 32);
        const float4* b4 = reinterpret_cast<const float4*>(e.beta + cgroup * 64 + c * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 gg = __ldg(g4 + j), bb = __ldg(b4 + j);
          v[4 * j] = keep ? (v[4 * j] - mean) * rstd * gg.x + bb.x : 0.f;
          v[4 * j + 1] = keep ? (v[4 * j + 1] - mean) * rstd * gg.y + bb.y : 0.f;
          v[4 * j + 2] = keep ? (v[4 * j + 2] - mean) * rstd * gg.z + bb.z : 0.f;
          v[4 * j + 3] = keep ? (v[4 * j + 3] - mean) * rstd * gg.w + bb.w : 0.f;
        }
        uint32_t packed[16];
        pack_bf16x32(v, packed);
        stage_row_chunks(stage, lane, c, packed);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(out_done);    // the GEMM 2 accumulator is drained
      fence_async_shared();
      __syncwarp();
      if (lane == 0) tma_store_2d(&tm_out, stage, cgroup * 64, m0 + quarter * 32);
      // every warp is past its statistics before the next tile writes the
      // LayerNorm partials again
      epilogue_sync();
    }
    if (lane == 0) tma_store_wait_all();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 0 && !*drain_failed) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && (*failed || *drain_failed)) set_status(e.status, GRS_ERR_TIMEOUT);
}

}  // namespace grs

extern "C" int grs_graph_mlp_bf16(const void* a, int64_t lda, const void* u0, int64_t ldu0,
                                  const float* b0, const void* u2, int64_t ldu2, const float* b2,
                                  int M, const void* residual, int64_t ldr, const float* gamma,
                                  const float* beta, const uint8_t* zero_row, float eps,
                                  void* out, int64_t ldo, int32_t* status, void* stream) {
  if (M <= 0) return GRS_OK;
  if (lda % 8 || ldu0 % 8 || ldu2 % 8 || ldr % 8 || ldo % 8 || lda < 512 || ldu0 < 512 ||
      ldu2 < 512 || ldr < 256 || ldo < 256)
    return GRS_ERR_SHAPE;
  if (!aligned16(a) || !aligned16(u0) || !aligned16(u2) || !aligned16(b0) || !aligned16(b2) ||
      !aligned16(residual) || !aligned16(gamma) || !aligned16(beta) || !aligned16(out) ||
      !b0 || !b2 || !residual || !gamma || !beta)
    return GRS_ERR_SHAPE;
  CUtensorMap tm_a, tm_u0, tm_u2, tm_res, tm_out;
  if (!gemm_map(&tm_a, a, M, 512, lda, GT_BM) || !gemm_map(&tm_u0, u0, 512, 512, ldu0, 256) ||
      !gemm_map(&tm_u2, u2, 256, 512, ldu2, 256) || !gemm_map(&tm_res, residual, M, 256, ldr, GT_BM) ||
      !gemm_map(&tm_out, out, M, 256, ldo, 32))
    return GRS_ERR_SHAPE;
  static bool attr[64] = {};
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(graph_mlp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             GM_SMEM) != cudaSuccess)
      return GRS_ERR_CUDA;
    attr[dev] = true;
  }
  if (dev < 64 && !sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int tiles = (M + GT_BM - 1) / GT_BM;
  const int grid = std::min(tiles, dev < 64 && sms[dev] ? sms[dev] : 148);
  GraphMlpArgs e{b0, b2, gamma, beta, zero_row, eps, status};
  graph_mlp_kernel<<<grid, GM_THREADS, GM_SMEM, counted((cudaStream_t)stream)>>>(
      tm_a, tm_u0, tm_u2, tm_res, tm_out, M, e);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}
