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
};

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
  } else {  // epilogue warps: TMEM -> registers -> bias, GELU -> bf16 -> smem -> TMA store
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
        if (e.bias) {
          const float4* b4 = reinterpret_cast<const float4*>(e.bias + n0 + col);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 bb = __ldg(b4 + j);
            v[4 * j] += bb.x;
            v[4 * j + 1] += bb.y;
            v[4 * j + 2] += bb.z;
            v[4 * j + 3] += bb.w;
          }
        }
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float2 p = make_float2(v[2 * j], v[2 * j + 1]);
          if (e.gelu) p = gelu_pair(p);
          __nv_bfloat162 h = __floats2bfloat162_rn(p.x, p.y);
          packed[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        // row `lane` of the block, 16-byte chunks placed by the 128-byte
        // swizzle the output tensor map uses (chunk ^ row % 8)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int chunk = c * 4 + j;
          *reinterpret_cast<uint4*>(stage + lane * 128 + ((chunk ^ (lane & 7)) << 4)) =
              make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
        }
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

extern "C" int grs_gemm_bf16_epilogue(const void* a, int64_t lda, const void* b, int64_t ldb,
                                      int M, int N, int K, const float* bias, int gelu,
                                      void* out, int64_t ldo, int32_t* status, void* stream) {
  if (M <= 0 || N <= 0 || K <= 0 || K % GT_BK || N % GT_BN || lda % 8 || ldb % 8 || ldo % 8 ||
      lda < K || ldb < K || ldo < N)
    return GRS_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
       reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(bias)) & 15)
    return GRS_ERR_SHAPE;
  CUtensorMap tm_a, tm_b, tm_out;
  if (!gemm_map(&tm_a, a, M, K, lda, GT_BM) || !gemm_map(&tm_b, b, N, K, ldb, GT_BN) ||
      !gemm_map(&tm_out, out, M, N, ldo, 32))
    return GRS_ERR_SHAPE;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GT_SMEM);
    attr[dev] = true;
  }
  GemmEpilogue e{bias, gelu, static_cast<__nv_bfloat16*>(out), ldo, status};
  static int sms[64] = {};
  if (dev < 64 && !sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int64_t tiles = (int64_t)((M + GT_BM - 1) / GT_BM) * (N / GT_BN);
  const int grid = (int)std::min<int64_t>(tiles, dev < 64 && sms[dev] ? sms[dev] : 148);
  gemm_tc_kernel<<<grid, GT_THREADS, GT_SMEM, counted((cudaStream_t)stream)>>>(tm_a, tm_b, tm_out,
                                                                               M, N, K, e);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}
