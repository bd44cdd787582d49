// bf16 GEMM with a fused row epilogue on the 5th-generation tensor cores:
//   out[M, N] = epilogue(A[M, K] . B[N, K]^T),  epilogue = (+ bias[N]) (GELU)
// A is row-major with row stride lda, B is K-major (a PyTorch Linear weight
// [out, in]), fp32 accumulation in tensor memory.  It replaces the cuBLAS
// GEMM followed by a separate bias+GELU pass of the readout graph layers
// (paged_model.py:381-436, model.py:26-53: the u0 projection and its GELU),
// so the [M, N] product is written once instead of written, read and
// written again.
//
// Persistent and warp-specialised, one CTA per SM walking 128 x 256 output
// tiles (consecutive tiles share their A rows): warp 0 (one thread) streams
// 64-wide K slices of A and B with TMA into a three-stage ring (128-byte
// swizzle); warp 1 (one thread) issues tcgen05.mma into one of two 256-column
// fp32 accumulators in TMEM and commits each stage back to the producer and
// each finished tile to the epilogue; warps 2-17 drain the other accumulator
// meanwhile (warp w reads TMEM lanes 32 (w % 4), columns 64 ((w - 2) / 4)),
// apply bias and GELU, stage the bf16 block in shared memory with the
// 128-byte swizzle and write it with a TMA store.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "grs_common.cuh"
#include "sm100.cuh"

namespace grs {

constexpr int GT_BM = 128, GT_BN = 256, GT_BK = 64, GT_STAGES = 3, GT_ACC = 2;
constexpr int GT_EPI_WARPS = 16, GT_THREADS = (2 + GT_EPI_WARPS) * 32;
constexpr int GT_A_BYTES = GT_BM * GT_BK * 2;                 // 16 KB
constexpr int GT_B_BYTES = GT_BN * GT_BK * 2;                 // 32 KB
constexpr int GT_STAGE_BYTES = GT_A_BYTES + GT_B_BYTES;
constexpr int GT_OUT_BYTES = 32 * 128;                        // one warp's 32 x 64 bf16 block
constexpr int GT_SMEM = GT_STAGES * GT_STAGE_BYTES + GT_EPI_WARPS * GT_OUT_BYTES +
                        1024;                                 // + 1024-byte alignment slack

struct GemmEpilogue {
  const float* bias;        // [N] or null
  int gelu;
  __nv_bfloat16* out;
  int64_t ldo;
  int32_t* status;
  // residual + LayerNorm epilogue (N == 256: a whole row per tile)
  const __nv_bfloat16* residual;
  int64_t ldr;
  const float* gamma;
  const float* beta;
  const uint8_t* zero_row;  // rows whose output is zeroed, or null
  float eps;
};

// named barrier of the four epilogue warps that share one TMEM lane quarter
__device__ __forceinline__ void quarter_sync(int quarter) {
  asm volatile("bar.sync %0, 128;\n" ::"r"(1 + quarter) : "memory");
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
  const float ex = __fdividef(1.f, q.x), ey = __fdividef(1.f, q.y);
  return make_float2(x.x >= 0.f ? x.x * fmaf(-0.5f, ex, 1.f) : 0.5f * x.x * ex,
                     x.y >= 0.f ? x.y * fmaf(-0.5f, ey, 1.f) : 0.5f * x.y * ey);
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

// Epilogue modes: bias (+ GELU); or bias + residual + LayerNorm over the
// 256-column row (+ zeroing of masked rows).
constexpr int GT_EPI_GELU = 0, GT_EPI_LAYERNORM = 1;

template <int MODE>
__global__ void __launch_bounds__(GT_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
               const __grid_constant__ CUtensorMap tm_out, int M, int N, int K, GemmEpilogue e) {
  using namespace sm100;
  extern __shared__ uint8_t gt_smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[GT_STAGES], empty_bar[GT_STAGES];
  __shared__ __align__(8) uint64_t tmem_full[GT_ACC], tmem_empty[GT_ACC];
  __shared__ uint32_t tmem_slot;
  __shared__ int failed;
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(gt_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k_iters = K / GT_BK;
  const int n_tiles = N / GT_BN;
  const int tiles = ((M + GT_BM - 1) / GT_BM) * n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < GT_STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < GT_ACC; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], GT_EPI_WARPS);
    }
    failed = 0;
    mbar_init_fence();
  }
  if (warp == 0) tmem_alloc(&tmem_slot, GT_ACC * GT_BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer: the ring runs across tiles
      int g = 0;
      for (int t = blockIdx.x; t < tiles && !failed; t += gridDim.x) {
        const int m0 = (t / n_tiles) * GT_BM, n0 = (t % n_tiles) * GT_BN;
        for (int it = 0; it < k_iters; ++it, ++g) {
          const int s = g % GT_STAGES, r = g / GT_STAGES;
          if (r > 0 && !mbar_wait(&empty_bar[s], (r - 1) & 1)) {
            failed = 1;
            break;
          }
          uint8_t* a = smem + s * GT_STAGE_BYTES;
          mbar_arrive_expect_tx(&full_bar[s], GT_STAGE_BYTES);
          tma_load_2d(a, &tm_a, it * GT_BK, m0, &full_bar[s]);
          tma_load_2d(a + GT_A_BYTES, &tm_b, it * GT_BK, n0, &full_bar[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      constexpr uint32_t idesc = idesc_bf16_f32(GT_BM, GT_BN);
      int g = 0, i = 0;
      for (int t = blockIdx.x; t < tiles && !failed; t += gridDim.x, ++i) {
        const int b = i & 1, u = i >> 1;
        if (u > 0 && !mbar_wait(&tmem_empty[b], (u - 1) & 1)) {
          failed = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * GT_BN);
        for (int it = 0; it < k_iters; ++it, ++g) {
          const int s = g % GT_STAGES, r = g / GT_STAGES;
          if (!mbar_wait(&full_bar[s], r & 1)) {
            failed = 1;
            break;
          }
          tc_fence_after();
          const uint8_t* a = smem + s * GT_STAGE_BYTES;
          const uint64_t ad = smem_desc_k128(a), bd = smem_desc_k128(a + GT_A_BYTES);
#pragma unroll
          for (int kk = 0; kk < GT_BK / 16; ++kk)  // 16 bf16 = 32 bytes = 2 descriptor units
            mma_bf16(acc, ad + 2 * kk, bd + 2 * kk, idesc, it > 0 || kk > 0);
          mma_commit(&empty_bar[s]);
        }
        mma_commit(&tmem_full[b]);
      }
    }
  } else if (MODE == GT_EPI_GELU) {
    // epilogue warps: TMEM -> registers -> bias, GELU -> bf16 -> smem -> TMA store
    const int quarter = warp & 3, cgroup = (warp - 2) >> 2;   // 64 columns per warp
    uint8_t* stage = smem + GT_STAGES * GT_STAGE_BYTES + (warp - 2) * GT_OUT_BYTES;
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int m0 = (t / n_tiles) * GT_BM, n0 = (t % n_tiles) * GT_BN;
      const int b = i & 1, u = i >> 1;
      if (!mbar_wait(&tmem_full[b], u & 1)) {
        failed = 1;
        break;
      }
      tc_fence_after();
      if (lane == 0) tma_store_wait_read();   // this warp's previous block has left smem
      __syncwarp();
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        const int col = cgroup * 64 + c * 32;
        float v[32];
        tmem_load32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * GT_BN + col), v);
        if (e.bias) add_bias32(v, e.bias + n0 + col);
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float2 p = make_float2(v[2 * j], v[2 * j + 1]);
          if (e.gelu) p = gelu_pair(p);
          __nv_bfloat162 h = __floats2bfloat162_rn(p.x, p.y);
          packed[j] = *reinterpret_cast<uint32_t*>(&h);
        }
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
  } else {
    // epilogue warps, LayerNorm mode: each row's 256 columns are spread over
    // the four warps of its lane quarter; per-warp (mean, centred sum of
    // squares) pairs meet in shared memory and merge exactly, so one pass
    // over the accumulator gives the statistics and a second writes the row
    __shared__ float ln_part[4][4][32], ln_m2[4][4][32];
    const int quarter = warp & 3, cgroup = (warp - 2) >> 2;
    uint8_t* stage = smem + GT_STAGES * GT_STAGE_BYTES + (warp - 2) * GT_OUT_BYTES;
    int i = 0;
    bool gave_up = false;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int m0 = t * GT_BM;                                 // N == 256: one tile per row block
      const int b = i & 1, u = i >> 1;
      // after a wait gave up, the warp still runs every named barrier so the
      // other warps of its quarter are not left waiting
      if (!gave_up && !mbar_wait(&tmem_full[b], u & 1)) {
        gave_up = true;
        failed = 1;
      }
      tc_fence_after();
      if (lane == 0) tma_store_wait_read();
      __syncwarp();
      const int row = m0 + quarter * 32 + lane;
      const bool in = row < M;
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * GT_BN);
      // v = acc + bias + residual for one 32-column chunk
      const auto load_row = [&](int c, float v[32]) {
        const int col = cgroup * 64 + c * 32;
        tmem_load32(taddr + (uint32_t)col, v);
        add_bias32(v, e.bias + col);
        if (in) {
          const uint4* x4 = reinterpret_cast<const uint4*>(e.residual + (int64_t)row * e.ldr + col);
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
      quarter_sync(quarter);
      // the row's four 64-column groups, merged pairwise the same way
      const float* pm = &ln_part[quarter][0][lane];
      const float* p2 = &ln_m2[quarter][0][lane];
      const float d01 = pm[32] - pm[0], d23 = pm[96] - pm[64];
      const float mean01 = pm[0] + 0.5f * d01, mean23 = pm[64] + 0.5f * d23;
      const float m201 = p2[0] + p2[32] + 32.f * d01 * d01;
      const float m223 = p2[64] + p2[96] + 32.f * d23 * d23;
      const float dd = mean23 - mean01;
      const float mean = mean01 + 0.5f * dd;
      const float var = (m201 + m223 + 64.f * dd * dd) * (1.f / GT_BN);
      quarter_sync(quarter);
      const float rstd = rsqrtf(var + e.eps);
      const bool keep = !in || e.zero_row == nullptr || e.zero_row[row] != 0;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        const int col = cgroup * 64 + c * 32;
        float v[32];
        load_row(c, v);
        uint32_t packed[16];
        const float4* g4 = reinterpret_cast<const float4*>(e.gamma + col);
        const float4* b4 = reinterpret_cast<const float4*>(e.beta + col);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 g = __ldg(g4 + j), bb = __ldg(b4 + j);
          float r[4] = {(v[4 * j] - mean) * rstd * g.x + bb.x,
                        (v[4 * j + 1] - mean) * rstd * g.y + bb.y,
                        (v[4 * j + 2] - mean) * rstd * g.z + bb.z,
                        (v[4 * j + 3] - mean) * rstd * g.w + bb.w};
          if (!keep) r[0] = r[1] = r[2] = r[3] = 0.f;
          __nv_bfloat162 h0 = __floats2bfloat162_rn(r[0], r[1]);
          __nv_bfloat162 h1 = __floats2bfloat162_rn(r[2], r[3]);
          packed[2 * j] = *reinterpret_cast<uint32_t*>(&h0);
          packed[2 * j + 1] = *reinterpret_cast<uint32_t*>(&h1);
        }
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
    if (lane == 0) tma_store_wait_all();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, GT_ACC * GT_BN);
  }
  if (threadIdx.x == 0 && failed) set_status(e.status, GRS_ERR_TIMEOUT);
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
// columns x box_rows rows, 128-byte swizzle; a small cache keyed by every
// encoded field.
bool gemm_map(CUtensorMap* out, const void* base, int64_t rows, int64_t cols, int64_t ld,
              int box_rows) {
  struct Key { const void* base; int64_t rows, cols, ld; int box; };
  constexpr int kCache = 32;
  static Key keys[kCache];
  static CUtensorMap maps[kCache];
  static int used = 0, next = 0;
  static std::mutex mu;
  Key k;
  std::memset(&k, 0, sizeof(k));
  k.base = base; k.rows = rows; k.cols = cols; k.ld = ld; k.box = box_rows;
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
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows}, estr[2] = {1, 1};
  CUtensorMap m;
  if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), gdim, gstr, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  keys[next] = k;
  maps[next] = m;
  next = (next + 1) % kCache;
  used = used < kCache ? used + 1 : kCache;
  *out = m;
  return true;
}

}  // namespace
}  // namespace grs

using namespace grs;

namespace grs {
namespace {

int launch_gemm(int mode, const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N,
                int K, void* out, int64_t ldo, const GemmEpilogue& e, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || K % GT_BK || N % GT_BN || lda % 8 || ldb % 8 || ldo % 8 ||
      lda < K || ldb < K || ldo < N)
    return GRS_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
       reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(e.bias)) & 15)
    return GRS_ERR_SHAPE;
  CUtensorMap tm_a, tm_b, tm_out;
  if (!gemm_map(&tm_a, a, M, K, lda, GT_BM) || !gemm_map(&tm_b, b, N, K, ldb, GT_BN) ||
      !gemm_map(&tm_out, out, M, N, ldo, 32))
    return GRS_ERR_SHAPE;
  static bool attr[2][64] = {};
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[mode][dev]) {
    cudaFuncSetAttribute(mode == GT_EPI_GELU ? gemm_tc_kernel<GT_EPI_GELU>
                                             : gemm_tc_kernel<GT_EPI_LAYERNORM>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, GT_SMEM);
    attr[mode][dev] = true;
  }
  if (dev < 64 && !sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int64_t tiles = (int64_t)((M + GT_BM - 1) / GT_BM) * (N / GT_BN);
  const int grid = (int)std::min<int64_t>(tiles, dev < 64 && sms[dev] ? sms[dev] : 148);
  if (mode == GT_EPI_GELU)
    gemm_tc_kernel<GT_EPI_GELU><<<grid, GT_THREADS, GT_SMEM, counted(stream)>>>(
        tm_a, tm_b, tm_out, M, N, K, e);
  else
    gemm_tc_kernel<GT_EPI_LAYERNORM><<<grid, GT_THREADS, GT_SMEM, counted(stream)>>>(
        tm_a, tm_b, tm_out, M, N, K, e);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

}  // namespace
}  // namespace grs

extern "C" int grs_gemm_bf16_epilogue(const void* a, int64_t lda, const void* b, int64_t ldb,
                                      int M, int N, int K, const float* bias, int gelu,
                                      void* out, int64_t ldo, int32_t* status, void* stream) {
  GemmEpilogue e{bias, gelu, static_cast<__nv_bfloat16*>(out), ldo, status,
                 nullptr, 0, nullptr, nullptr, nullptr, 0.f};
  return launch_gemm(GT_EPI_GELU, a, lda, b, ldb, M, N, K, out, ldo, e, (cudaStream_t)stream);
}

extern "C" int grs_gemm_bf16_layernorm(const void* a, int64_t lda, const void* b, int64_t ldb,
                                       int M, int K, const float* bias, const void* residual,
                                       int64_t ldr, const float* gamma, const float* beta,
                                       const uint8_t* zero_row, float eps, void* out,
                                       int64_t ldo, int32_t* status, void* stream) {
  if (bias == nullptr || residual == nullptr || gamma == nullptr || beta == nullptr ||
      ldr % 8 || (reinterpret_cast<uintptr_t>(residual) & 15) ||
      (reinterpret_cast<uintptr_t>(gamma) & 15) || (reinterpret_cast<uintptr_t>(beta) & 15))
    return GRS_ERR_SHAPE;
  GemmEpilogue e{bias, 0, static_cast<__nv_bfloat16*>(out), ldo, status,
                 static_cast<const __nv_bfloat16*>(residual), ldr, gamma, beta, zero_row, eps};
  return launch_gemm(GT_EPI_LAYERNORM, a, lda, b, ldb, M, GT_BN, K, out, ldo, e,
                     (cudaStream_t)stream);
}
