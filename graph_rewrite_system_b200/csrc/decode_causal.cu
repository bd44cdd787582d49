// One-token causal decode over paged K/V: the attention of the causal action
// layers (paged_model.py:66-94), i.e. paged_attention with one query per
// (beam, head) over the first lengths[b] tokens of the beam's block-table
// pages plus, when current_valid[b], the current token at position
// lengths[b] (paged_attention.py:18-159, current token :101-132).  bf16,
// head width 32.
//
// One CTA per beam, one warp per head.  Thread 0 stages the beam's pages in
// 64-token chunks into shared memory with one 1-D bulk copy (TMA) per page of
// K and of V - a page of `page` tokens x heads x 32 bf16 is one contiguous
// block of the arena - completing on an mbarrier (bounded wait).  Each warp
// then scores its head lane-per-token (the token's 64-byte key row read as
// four 16-byte pieces in a lane-rotated order, at most 2-way bank conflicts),
// merges the chunk into an fp32 online softmax and accumulates P.V
// lane-per-dimension (one contiguous 64-byte value row per token).  The
// current token joins as one more key.  Rows with no valid key are zero;
// page ids outside the arena flag GRS_ERR_BAD_PAGE and their tokens are
// skipped.
#include "grs_common.cuh"
#include "sm100.cuh"

namespace grs {

constexpr int DP_D = 32;          // head width
constexpr int DP_CHUNK = 64;      // tokens staged per chunk
constexpr int DP_MAX_HEADS = 16;

struct DecodeCausalArgs {
  const __nv_bfloat16* q; int64_t q_sb, q_sh;
  const __nv_bfloat16* kc; const __nv_bfloat16* vc; int64_t kc_sp;
  const int32_t* bt; int64_t bt_s; const int32_t* lengths; int num_pages;
  const __nv_bfloat16* ck; const __nv_bfloat16* cv; int64_t ck_sb, ck_sh;
  const uint8_t* cvalid;
  __nv_bfloat16* out; int64_t o_sb, o_sh;
  int heads, page;
  float scale_log2;
  int32_t* status;
};

__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
      ::"r"(sm100::smem_u32(dst)), "l"(src), "r"(bytes), "r"(sm100::smem_u32(bar))
      : "memory");
}

// The 32 bf16 of one head row (64 bytes, 16-byte aligned) as fp32, read as
// four 16-byte pieces starting at piece `rot`: v[8 j + i] = row[8 ((j + rot)
// mod 4) + i].  Registers are indexed statically; only the addresses rotate.
__device__ __forceinline__ void load_row32(const __nv_bfloat16* src, int rot, float v[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 w = *reinterpret_cast<const uint4*>(src + ((j + rot) & 3) * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __bfloat1622float2(h[k]);
      v[8 * j + 2 * k] = f.x;
      v[8 * j + 2 * k + 1] = f.y;
    }
  }
}

__device__ __forceinline__ float dot32(const float a[32], const float b[32]) {
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int d = 0; d < 32; d += 2) {
    s0 = fmaf(a[d], b[d], s0);
    s1 = fmaf(a[d + 1], b[d + 1], s1);
  }
  return s0 + s1;
}

__global__ void __launch_bounds__(DP_MAX_HEADS * 32, 1) decode_causal_kernel(DecodeCausalArgs a) {
  using namespace sm100;
  extern __shared__ __align__(128) uint8_t dc_smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint8_t page_ok[DP_CHUNK];
  const int b = blockIdx.x;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_elems = a.heads * DP_D;                 // one token of all heads
  const uint32_t page_bytes = (uint32_t)a.page * row_elems * 2;
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(dc_smem);
  __nv_bfloat16* vs = ks + DP_CHUNK * row_elems;
  const int past = a.lengths[b];

  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_init_fence();
  }
  __syncthreads();

  // this head's query, pre-scaled by log2(e) / sqrt(32), in every lane,
  // rotated like this lane's key reads
  const int rot = lane & 3;
  float qr[32];
  load_row32(a.q + (int64_t)b * a.q_sb + (int64_t)h * a.q_sh, rot, qr);
#pragma unroll
  for (int d = 0; d < 32; ++d) qr[d] *= a.scale_log2;

  float m = -1e30f, l = 0.f, acc = 0.f;       // lane owns output dimension `lane`
  bool ok = true;
  int phase = 0;
  for (int c0 = 0; c0 < past; c0 += DP_CHUNK) {
    const int n = min(DP_CHUNK, past - c0);
    const int np = (n + a.page - 1) / a.page;
    if (threadIdx.x == 0) {
      const int32_t* row = a.bt + (int64_t)b * a.bt_s + c0 / a.page;
      uint32_t bytes = 0;
      bool bad = false;
      for (int p = 0; p < np; ++p) {
        const int pid = row[p];
        const bool valid = pid >= 0 && pid < a.num_pages;
        page_ok[p] = valid;
        bad |= !valid;
        bytes += valid ? 2 * page_bytes : 0;
      }
      mbar_arrive_expect_tx(&bar, bytes);
      for (int p = 0; p < np; ++p) {
        if (!page_ok[p]) continue;
        const int64_t off = (int64_t)row[p] * a.kc_sp;
        bulk_copy_g2s(ks + (size_t)p * a.page * row_elems, a.kc + off, page_bytes, &bar);
        bulk_copy_g2s(vs + (size_t)p * a.page * row_elems, a.vc + off, page_bytes, &bar);
      }
      if (bad) set_status(a.status, GRS_ERR_BAD_PAGE);
    }
    const bool arrived = mbar_wait(&bar, phase & 1);
    ++phase;
    if (!__syncthreads_and(arrived)) {
      // the copies of this chunk did not land in time: wait once more for
      // them (bounded) so none is in flight when the CTA exits, report, stop
      if (threadIdx.x == 0) {
        mbar_wait(&bar, (phase - 1) & 1);
        set_status(a.status, GRS_ERR_TIMEOUT);
      }
      ok = false;
      break;
    }
    // scores of the chunk: lane-per-token (tokens lane and lane + 32)
    float s[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int t = lane + 32 * i;
      s[i] = -INFINITY;
      if (t < n && page_ok[t / a.page]) {
        float k[32];
        load_row32(ks + (size_t)t * row_elems + h * DP_D, rot, k);
        s[i] = dot32(qr, k);
      }
    }
    const float m_new = fmaxf(m, warp_max(fmaxf(s[0], s[1])));
    const float corr = exp2f(m - m_new);
    const float p0 = exp2f(s[0] - m_new), p1 = exp2f(s[1] - m_new);
    l = l * corr + warp_sum(p0 + p1);
    acc *= corr;
    m = m_new;
    // P.V lane-per-dimension
    const __nv_bfloat16* vrow = vs + h * DP_D + lane;
    int t = 0;
    for (; t + 4 <= n; t += 4) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int tt = t + u;
        const float pt = __shfl_sync(0xffffffffu, tt < 32 ? p0 : p1, tt & 31);
        acc = fmaf(pt, __bfloat162float(vrow[(size_t)tt * row_elems]), acc);
      }
    }
    for (; t < n; ++t) {
      const float pt = __shfl_sync(0xffffffffu, t < 32 ? p0 : p1, t & 31);
      acc = fmaf(pt, __bfloat162float(vrow[(size_t)t * row_elems]), acc);
    }
    __syncthreads();                 // the next chunk overwrites the stage
  }
  __nv_bfloat16* op = a.out + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh;
  if (!ok) {
    op[lane] = __float2bfloat16_rn(0.f);
    return;
  }
  if (a.ck != nullptr && (a.cvalid == nullptr || a.cvalid[b] != 0)) {
    float k[32];
    const int64_t off = (int64_t)b * a.ck_sb + (int64_t)h * a.ck_sh;
    load_row32(a.ck + off, rot, k);
    const float sc = dot32(qr, k);
    const float m_new = fmaxf(m, sc);
    const float corr = exp2f(m - m_new);
    const float pc = exp2f(sc - m_new);
    l = l * corr + pc;
    acc = fmaf(pc, __bfloat162float(a.cv[off + lane]), acc * corr);
  }
  op[lane] = __float2bfloat16_rn(l > 0.f ? acc / l : 0.f);
}

}  // namespace grs

using namespace grs;

extern "C" int grs_decode_causal(const void* query, int64_t q_sb, int64_t q_sh,
                                 const void* key_cache, const void* value_cache, int64_t kc_sp,
                                 int64_t kc_st, int64_t kc_sh, const int32_t* block_table,
                                 int64_t bt_s, const int32_t* lengths, int num_pages,
                                 const void* current_key, const void* current_value,
                                 int64_t ck_sb, int64_t ck_sh, const uint8_t* current_valid,
                                 void* out, int64_t o_sb, int64_t o_sh, int batch, int heads,
                                 int page, int32_t* status, void* stream) {
  if (batch <= 0) return GRS_OK;
  if (heads <= 0 || heads > DP_MAX_HEADS || page <= 0 || DP_CHUNK % page) return GRS_ERR_SHAPE;
  const int64_t row = (int64_t)heads * DP_D;
  if (kc_sh != DP_D || kc_st != row || kc_sp != page * row) return GRS_ERR_SHAPE;
  if (((uintptr_t)query | (uintptr_t)key_cache | (uintptr_t)value_cache) & 15) return GRS_ERR_SHAPE;
  if ((q_sb | q_sh) % 8) return GRS_ERR_SHAPE;
  if (current_key != nullptr &&
      ((((uintptr_t)current_key | (uintptr_t)current_value) & 15) || (ck_sb | ck_sh) % 8))
    return GRS_ERR_SHAPE;
  if (((uintptr_t)out & 1) || !block_table || !lengths) return GRS_ERR_SHAPE;
  DecodeCausalArgs a;
  a.q = static_cast<const __nv_bfloat16*>(query); a.q_sb = q_sb; a.q_sh = q_sh;
  a.kc = static_cast<const __nv_bfloat16*>(key_cache);
  a.vc = static_cast<const __nv_bfloat16*>(value_cache);
  a.kc_sp = kc_sp;
  a.bt = block_table; a.bt_s = bt_s; a.lengths = lengths; a.num_pages = num_pages;
  a.ck = static_cast<const __nv_bfloat16*>(current_key);
  a.cv = static_cast<const __nv_bfloat16*>(current_value);
  a.ck_sb = ck_sb; a.ck_sh = ck_sh; a.cvalid = current_valid;
  a.out = static_cast<__nv_bfloat16*>(out); a.o_sb = o_sb; a.o_sh = o_sh;
  a.heads = heads; a.page = page;
  a.scale_log2 = 1.4426950408889634f / sqrtf((float)DP_D);
  a.status = status;
  const size_t smem = (size_t)2 * DP_CHUNK * row * 2;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(decode_causal_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             2 * DP_CHUNK * DP_MAX_HEADS * DP_D * 2) != cudaSuccess)
      return GRS_ERR_CUDA;
    attr[dev] = true;
  }
  decode_causal_kernel<<<batch, heads * 32, smem, counted((cudaStream_t)stream)>>>(a);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}
