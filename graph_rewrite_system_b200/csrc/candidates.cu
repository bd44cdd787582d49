// Candidate selection and structural binding decode (reference
// threshold_inference.py:208-297, model.py:391-478).
//
// select_candidates: one CTA per beam row.  Every (slot, source) pair whose
// raw logit passes the near/far threshold and is eligible gets the
// calibrated score logit * scale + bias (two roundings, as the reference's
// separate multiply and add); the K best scores (ties: lower flat index) are
// found with a 4 x 8-bit MSB radix select over order-preserving score bits in
// shared-memory histograms, then sorted by (score desc, index asc) with a
// shared-memory bitonic sort.  Output rows are padded to K with source -1.
//
// structural_decode: one thread per candidate follows the source pattern's
// port edges from the anchor through the per-beam port arrays and verifies
// every pattern edge; invalid candidates can be cleared (source -1) so the
// padded candidate arrays feed the proposal ranking without compaction.
#include "grs_common.cuh"

namespace grs {

constexpr int SEL_THREADS = 512;
constexpr int SEL_MAX_K = 2048;

__device__ __forceinline__ uint32_t float_order(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float order_float(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

struct SelectArgs {
  const float* logits;           // [B, S, ns]
  const uint8_t* eligible;       // [B, S, ns]
  const int32_t* distance;       // [B, S]
  int slots, num_sources, k;
  float near_scale, near_bias, near_thr, far_scale, far_bias, far_thr;
  int64_t* out_batch; int64_t* out_source; int64_t* out_anchor; float* out_prob;
  float* out_score;              // optional calibrated score
  int vec8;                      // rows are whole 8-item chunks, 16-byte aligned
};

// the item's key from its already loaded eligibility and logit
__device__ __forceinline__ bool item_key_loaded(const SelectArgs& a, int64_t row, int idx,
                                                bool eligible, float logit, uint32_t* key) {
  if (!eligible) return false;
  const int slot = idx / a.num_sources;
  const bool near = a.distance[row * a.slots + slot] <= 2;
  const float thr = near ? a.near_thr : a.far_thr;
  if (!(logit >= thr)) return false;
  const float calibrated = __fadd_rn(__fmul_rn(logit, near ? a.near_scale : a.far_scale),
                                     near ? a.near_bias : a.far_bias);
  if (!(calibrated > -INFINITY)) return false;  // -inf scores are not present
  *key = float_order(calibrated);
  return true;
}

__device__ __forceinline__ bool item_key(const SelectArgs& a, int64_t row, int idx,
                                         uint32_t* key) {
  const int64_t off = row * (int64_t)a.slots * a.num_sources + idx;
  if (!a.eligible[off]) return false;
  return item_key_loaded(a, row, idx, true, a.logits[off], key);
}

__global__ void __launch_bounds__(SEL_THREADS) select_candidates_kernel(SelectArgs a) {
  __shared__ int hist[256];
  __shared__ int s_bin, s_above, s_all, s_count, s_eq_base;
  __shared__ int warp_tot[SEL_THREADS / 32];
  __shared__ unsigned long long sel[SEL_MAX_K];
  const int64_t row = blockIdx.x;
  const int n = a.slots * a.num_sources;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t prefix = 0, mask = 0;
  int remaining = a.k;
  bool take_all = false;
  if (tid == 0) s_count = 0;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += SEL_THREADS) hist[i] = 0;
    __syncthreads();
    if (pass == 0 && a.vec8) {
      // 8-item chunks: a thread's eligibility bytes and logits arrive in one
      // 8-byte and two 16-byte loads
      const int64_t base = row * (int64_t)n;
      for (int ch = tid; ch < n / 8; ch += SEL_THREADS) {
        const int idx0 = ch * 8;
        const uint2 el = *reinterpret_cast<const uint2*>(a.eligible + base + idx0);
        const float4 l0 = *reinterpret_cast<const float4*>(a.logits + base + idx0);
        const float4 l1 = *reinterpret_cast<const float4*>(a.logits + base + idx0 + 4);
        const float lg[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const bool e = ((j < 4 ? el.x : el.y) >> (8 * (j & 3))) & 0xffu;
          uint32_t key;
          if (item_key_loaded(a, row, idx0 + j, e, lg[j], &key)) {
            atomicAdd(&hist[(key >> shift) & 255], 1);
            const int slot = atomicAdd(&s_count, 1);
            if (slot < SEL_MAX_K)
              sel[slot] = ((unsigned long long)key << 32) |
                          (unsigned long long)(0xffffffffu - (uint32_t)(idx0 + j));
          }
        }
      }
    }
    for (int idx = tid; !(pass == 0 && a.vec8) && idx < n; idx += SEL_THREADS) {
      uint32_t key;
      if (item_key(a, row, idx, &key) && (key & mask) == prefix) {
        atomicAdd(&hist[(key >> shift) & 255], 1);
        // the first pass also keeps every item it sees: when they are no
        // more than k (the usual case), that is the whole selection and no
        // collect pass is needed (the sort below orders them)
        if (pass == 0) {
          const int slot = atomicAdd(&s_count, 1);
          if (slot < SEL_MAX_K)
            sel[slot] = ((unsigned long long)key << 32) |
                        (unsigned long long)(0xffffffffu - (uint32_t)idx);
        }
      }
    }
    __syncthreads();
    if (tid == 0) {
      int above = 0, bin = -1, total = 0;
      for (int d = 0; d < 256; ++d) total += hist[d];
      for (int d = 255; d >= 0; --d) {
        if (above + hist[d] >= remaining) { bin = d; break; }
        above += hist[d];
      }
      s_bin = bin; s_above = above; s_all = (pass == 0 && total <= remaining) ? 1 : 0;
    }
    __syncthreads();
    if (s_all) { take_all = true; break; }
    remaining -= s_above;
    prefix |= (uint32_t)s_bin << shift;
    mask |= 255u << shift;
    __syncthreads();
  }
  // Collect: keys above the threshold key, plus the first `remaining` keys
  // equal to it in index order (block scan over the index-ordered chunks);
  // when every item is taken the first pass already collected them
  __syncthreads();
  if (!take_all && tid == 0) { s_count = 0; s_eq_base = 0; }
  __syncthreads();
  for (int base = 0; !take_all && base < n; base += SEL_THREADS) {
    const int idx = base + tid;
    uint32_t key = 0;
    const bool valid = idx < n && item_key(a, row, idx, &key);
    const bool gt = valid && (take_all || key > prefix);
    const bool eq = valid && !take_all && key == prefix;
    const unsigned ballot = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) warp_tot[warp] = __popc(ballot);
    __syncthreads();
    int before = s_eq_base;
    for (int w = 0; w < warp; ++w) before += warp_tot[w];
    before += __popc(ballot & ((1u << lane) - 1u));
    const bool take = gt || (eq && before < remaining);
    if (take) {
      const int slot = atomicAdd(&s_count, 1);
      if (slot < SEL_MAX_K)
        sel[slot] = ((unsigned long long)key << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
    }
    __syncthreads();
    if (tid == 0) {
      int tot = 0;
      for (int w = 0; w < SEL_THREADS / 32; ++w) tot += warp_tot[w];
      s_eq_base += tot;
    }
    __syncthreads();
  }
  const int count = min(s_count, a.k);
  int size = 1;
  while (size < count) size <<= 1;
  for (int i = count + tid; i < size; i += SEL_THREADS) sel[i] = 0ull;
  __syncthreads();
  // Bitonic sort, descending.
  for (int k2 = 2; k2 <= size; k2 <<= 1) {
    for (int j = k2 >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < size; i += SEL_THREADS) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long x = sel[i], y = sel[l];
          const bool desc = (i & k2) == 0;
          if (desc ? (x < y) : (x > y)) { sel[i] = y; sel[l] = x; }
        }
      }
      __syncthreads();
    }
  }
  for (int r = tid; r < a.k; r += SEL_THREADS) {
    const int64_t o = row * a.k + r;
    a.out_batch[o] = row;
    if (r < count) {
      const unsigned long long v = sel[r];
      const int idx = (int)(0xffffffffu - (uint32_t)(v & 0xffffffffu));
      const float score = order_float((uint32_t)(v >> 32));
      a.out_anchor[o] = idx / a.num_sources;
      a.out_source[o] = idx % a.num_sources;
      a.out_prob[o] = 1.f / (1.f + expf(-score));
      if (a.out_score) a.out_score[o] = score;
    } else {
      a.out_anchor[o] = 0;
      a.out_source[o] = -1;
      a.out_prob[o] = 0.f;
      if (a.out_score) a.out_score[o] = -INFINITY;
    }
  }
}

struct DecodeArgs {
  const int64_t* types; const uint8_t* live; int slots;
  const int32_t* out_node; const int32_t* out_port; const int32_t* in_node;
  const int32_t* in_port;                                  // [B, S, 4]
  const int64_t* source_types; const int64_t* source_lengths;  // [ns, P], [ns]
  const int64_t* child; const int64_t* parent; const int64_t* parent_port;
  const int64_t* child_port; const int64_t* direction;      // [ns, P]
  const int64_t* pattern_edges; int max_edges;              // [ns, E, 4]
  int max_pattern;
  const int64_t* batch_ids; int64_t* sources; const int64_t* anchors; int64_t count;
  int64_t* bindings; uint8_t* valid; int clear_invalid;
};

__global__ void structural_decode_kernel(DecodeArgs a) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= a.count) return;
  const int P = a.max_pattern;
  int64_t* bind = a.bindings + c * P;
  const int64_t src = a.sources[c];
  for (int p = 0; p < P; ++p) bind[p] = -1;
  if (src < 0) { a.valid[c] = 0; return; }
  const int64_t b = a.batch_ids[c];
  const int64_t anchor = a.anchors[c];
  bind[0] = anchor;
  const int64_t* st = a.source_types + src * P;
  const int64_t base = b * a.slots;
  bool ok = anchor >= 0 && anchor < a.slots && a.live[base + anchor] &&
            a.types[base + anchor] == st[0];
  const int64_t len = a.source_lengths[src];
  for (int step = 0; step < P - 1; ++step) {
    const bool act = len > step + 1;
    const int64_t cp = a.child[src * P + step], pp = a.parent[src * P + step];
    if (act && !(pp >= 0 && cp >= 0)) ok = false;
    int64_t pslot = bind[pp < 0 ? 0 : pp];
    if (pslot < 0) pslot = 0;
    const int64_t pport = a.parent_port[src * P + step] < 0 ? 0 : a.parent_port[src * P + step];
    const int64_t cport = a.child_port[src * P + step];
    const bool fwd = a.direction[src * P + step] > 0;
    const int64_t pidx = (base + pslot) * 4 + pport;
    const int64_t cand = fwd ? a.out_node[pidx] : a.in_node[pidx];
    const int64_t cand_port = fwd ? a.out_port[pidx] : a.in_port[pidx];
    bool pos_ok = cand >= 0 && cand_port == cport;
    const int64_t safe = cand < 0 ? 0 : cand;
    pos_ok = pos_ok && a.live[base + safe];
    pos_ok = pos_ok && a.types[base + safe] == st[cp < 0 ? 0 : cp];
    for (int p = 0; p < P; ++p) pos_ok = pos_ok && bind[p] != cand;
    if (act && !pos_ok) ok = false;
    if (act && cp >= 0) bind[cp] = cand;
  }
  for (int e = 0; e < a.max_edges; ++e) {
    const int64_t* pe = a.pattern_edges + (src * a.max_edges + e) * 4;
    if (pe[0] < 0) continue;
    int64_t sslot = bind[pe[0]];
    if (sslot < 0) sslot = 0;
    const int64_t dslot = bind[pe[1] < 0 ? 0 : pe[1]];
    const int64_t sp = pe[2] < 0 ? 0 : pe[2];
    const int64_t pidx = (base + sslot) * 4 + sp;
    if (a.out_node[pidx] != dslot || a.out_port[pidx] != pe[3]) ok = false;
  }
  a.valid[c] = ok;
  if (!ok && a.clear_invalid) a.sources[c] = -1;
}

}  // namespace grs

using namespace grs;

extern "C" int grs_select_candidates(const float* logits, const uint8_t* eligible,
                                     const int32_t* distance, int batch, int slots,
                                     int num_sources, int k, float near_scale, float near_bias,
                                     float near_thr, float far_scale, float far_bias,
                                     float far_thr, int64_t* out_batch, int64_t* out_source,
                                     int64_t* out_anchor, float* out_prob, float* out_score,
                                     void* stream) {
  if (batch <= 0) return GRS_OK;
  if (k <= 0 || k > SEL_MAX_K || slots <= 0 || num_sources <= 0) return GRS_ERR_SHAPE;
  const int64_t n = (int64_t)slots * num_sources;
  const int vec8 = n % 8 == 0 && (reinterpret_cast<uintptr_t>(eligible) & 7) == 0 &&
                   (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  SelectArgs a{logits, eligible, distance, slots, num_sources, k, near_scale, near_bias,
               near_thr, far_scale, far_bias, far_thr, out_batch, out_source, out_anchor,
               out_prob, out_score, vec8};
  select_candidates_kernel<<<batch, SEL_THREADS, 0, grs::counted((cudaStream_t)stream)>>>(a);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_structural_decode(
    const int64_t* types, const uint8_t* live, int slots, const int32_t* out_node,
    const int32_t* out_port, const int32_t* in_node, const int32_t* in_port,
    const int64_t* source_types, const int64_t* source_lengths, const int64_t* child,
    const int64_t* parent, const int64_t* parent_port, const int64_t* child_port,
    const int64_t* direction, const int64_t* pattern_edges, int max_edges, int max_pattern,
    const int64_t* batch_ids, int64_t* sources, const int64_t* anchors, int64_t count,
    int64_t* bindings, uint8_t* valid, int clear_invalid, void* stream) {
  if (count <= 0) return GRS_OK;
  if (max_pattern <= 0 || slots <= 0) return GRS_ERR_SHAPE;
  DecodeArgs a{types, live, slots, out_node, out_port, in_node, in_port, source_types,
               source_lengths, child, parent, parent_port, child_port, direction, pattern_edges,
               max_edges, max_pattern, batch_ids, sources, anchors, count, bindings, valid,
               clear_invalid};
  structural_decode_kernel<<<ceil_div(count, 128), 128, 0, grs::counted((cudaStream_t)stream)>>>(a);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}
