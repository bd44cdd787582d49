// Device-resident lazy topology: rewrite planning with XOR fingerprints,
// first-occurrence dedup, accept, and child materialisation with the BFS
// rewrite distance (reference lazy_rollout_benchmark.py:105-485 and the accept
// loop of paged_rollout_benchmark.py:1013-1046).
//
// Per beam the topology is a set of port arrays (out/in node and port, int32
// [B, S, 4], -1 = unconnected), the gate type of every slot (int64 [B, S],
// -1 = dead), touch steps, the previous-preferred flags and scalars.  The
// sequential accept loop is reproduced exactly: a proposal is accepted iff it
// is valid, its fingerprint was not seen in earlier steps, and it is the
// first valid proposal with that fingerprint in rank order; the first
// beam_size such proposals are kept and stably sorted by next gate count.
#include "grs_common.cuh"
#include "topology_table.cuh"

namespace grs {

constexpr uint64_t EMPTY_KEY = 0ull;
__device__ __forceinline__ uint64_t table_key(uint64_t fp) { return fp == EMPTY_KEY ? 1ull : fp; }

struct Ports {
  int32_t* out_node; int32_t* out_port; int32_t* in_node; int32_t* in_port;
};

struct PlanArgs {
  int64_t count_cap;                 // global_cap
  const int64_t* count;              // device: number of ranked proposals
  const int64_t* rows; const int64_t* xfers; const int64_t* next_gate;
  const int64_t* cand_batch; const int64_t* cand_bindings; int cand_pattern;
  const int32_t* table;
  const int64_t* types; Ports ports; int slots;
  const int32_t* next_slot; const uint64_t* fingerprint;
  uint8_t* valid; uint64_t* fp_out;
  int32_t* status;
};

__device__ __forceinline__ bool in_set(const int64_t* set, int n, int64_t v) {
  for (int i = 0; i < n; ++i) if (set[i] == v) return true;
  return false;
}

__global__ void topology_plan_kernel(PlanArgs a) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= a.count_cap) return;
  a.valid[j] = 0;
  a.fp_out[j] = 0;
  if (j >= *a.count) return;
  const int64_t row = a.rows[j];
  const int64_t x = a.xfers[j];
  const int64_t parent = a.cand_batch[row];
  const int32_t* tab = a.table + x * TAB_WIDTH;
  const int src_len = tab[TAB_SRC_LEN], dst_len = tab[TAB_DST_LEN];
  int64_t bind[TAB_MAXP];
  int nb = 0;
  for (int k = 0; k < a.cand_pattern; ++k) {
    const int64_t v = a.cand_bindings[row * a.cand_pattern + k];
    if (v >= 0) {
      if (nb >= TAB_MAXP) return;
      bind[nb++] = v;
    }
  }
  if (nb != src_len) return;  // "source pattern/binding length mismatch"
  const int64_t base = parent * a.slots;
  for (int k = 0; k < nb; ++k)
    if (bind[k] >= a.slots || a.types[base + bind[k]] < 0) return;  // non-live source slot
  const int32_t ns = a.next_slot[parent];
  // Destination slots at or past the current row width do not exist yet
  // (the children's rows are widened when they are materialised).
  for (int i = 0; i < dst_len; ++i)
    if (ns + i < a.slots && a.types[base + ns + i] >= 0) return;  // reuses a live slot
  uint64_t fp = a.fingerprint[parent];
  for (int k = 0; k < nb; ++k) fp ^= node_component(bind[k], a.types[base + bind[k]]);
  for (int i = 0; i < dst_len; ++i) fp ^= node_component(ns + i, tab[TAB_DST_TYPES + i]);
  // removed edges: every edge at a removed slot, once
  for (int k = 0; k < nb; ++k) {
    const int64_t v = bind[k];
    for (int p = 0; p < 4; ++p) {
      const int64_t pi = (base + v) * 4 + p;
      const int32_t o = a.ports.out_node[pi];
      if (o >= 0) fp ^= edge_component(v, o, p, a.ports.out_port[pi]);
      const int32_t in = a.ports.in_node[pi];
      if (in >= 0 && !in_set(bind, nb, in)) fp ^= edge_component(in, v, a.ports.in_port[pi], p);
    }
  }
  // added edges, wire by wire
  const int nw = tab[TAB_NWIRES];
  for (int w = 0; w < nw; ++w) {
    const int32_t* wr = tab + TAB_WIRES + w * 8;
    int64_t pred = -1, pred_port = -1, succ = -1, succ_port = -1;
    if (wr[0] >= 0) {
      const int64_t pi = (base + bind[wr[0]]) * 4 + wr[1];
      if (a.ports.in_node[pi] >= 0 && !in_set(bind, nb, a.ports.in_node[pi])) {
        pred = a.ports.in_node[pi]; pred_port = a.ports.in_port[pi];
      }
      const int64_t si = (base + bind[wr[2]]) * 4 + wr[3];
      if (a.ports.out_node[si] >= 0 && !in_set(bind, nb, a.ports.out_node[si])) {
        succ = a.ports.out_node[si]; succ_port = a.ports.out_port[si];
      }
    }
    if (wr[4] >= 0) {
      if (pred >= 0) fp ^= edge_component(pred, ns + wr[4], pred_port, wr[5]);
      if (succ >= 0) fp ^= edge_component(ns + wr[6], succ, wr[7], succ_port);
    } else if (pred >= 0 && succ >= 0) {
      fp ^= edge_component(pred, succ, pred_port, succ_port);
    }
  }
  const int nint = tab[TAB_NINT];
  for (int e = 0; e < nint; ++e) {
    const int32_t* ie = tab + TAB_INT + e * 4;
    fp ^= edge_component(ns + ie[0], ns + ie[1], ie[2], ie[3]);
  }
  a.valid[j] = 1;
  a.fp_out[j] = fp;
}

// Step-local first-occurrence table: fingerprint -> lowest proposal index.
__global__ void topology_first_kernel(const uint8_t* valid, const uint64_t* fp, int64_t n,
                                      uint64_t* keys, int32_t* first, int64_t capacity,
                                      int32_t* status) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n || !valid[j]) return;
  const uint64_t key = table_key(fp[j]);
  uint64_t h = mix64(key) & (capacity - 1);
  for (int64_t probe = 0; probe < capacity; ++probe, h = (h + 1) & (capacity - 1)) {
    const unsigned long long prev = atomicCAS(reinterpret_cast<unsigned long long*>(&keys[h]),
                                              EMPTY_KEY, key);
    if (prev == EMPTY_KEY || prev == key) {
      atomicMin(&first[h], (int32_t)j);
      return;
    }
  }
  set_status(status, GRS_ERR_WORKSPACE);
}

__device__ __forceinline__ int64_t table_find(const uint64_t* keys, int64_t capacity, uint64_t key) {
  uint64_t h = mix64(key) & (capacity - 1);
  for (int64_t probe = 0; probe < capacity; ++probe, h = (h + 1) & (capacity - 1)) {
    const uint64_t k = keys[h];
    if (k == key) return (int64_t)h;
    if (k == EMPTY_KEY) return -1;
  }
  return -1;
}

__global__ void topology_classify_kernel(const uint8_t* valid, const uint64_t* fp, int64_t n,
                                         const uint64_t* keys, const int32_t* first,
                                         int64_t capacity, const uint64_t* seen,
                                         int64_t seen_capacity, uint8_t* accept) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  uint8_t code = 0;  // 0 invalid, 1 duplicate, 2 acceptable
  if (valid[j]) {
    const uint64_t key = table_key(fp[j]);
    const int64_t h = table_find(keys, capacity, key);
    const bool is_first = h >= 0 && first[h] == (int32_t)j;
    const bool was_seen = table_find(seen, seen_capacity, key) >= 0;
    code = (is_first && !was_seen) ? 2 : 1;
  }
  accept[j] = code;
}

// One CTA: walk the classified proposals in rank order exactly like the
// sequential loop (stop after beam_size accepts), count attempted / invalid /
// duplicates, record accepted fingerprints in the seen set and stably sort
// the accepted proposals by next gate count.
constexpr int ACC_THREADS = 1024;
__global__ void __launch_bounds__(ACC_THREADS) topology_accept_kernel(
    const uint8_t* accept, const int64_t* count_ptr, int64_t cap, const uint64_t* fp,
    const int64_t* next_gate, int beam_size, uint64_t* seen, int64_t seen_capacity,
    int64_t* child_proposal, int64_t* summary, int32_t* status) {
  extern __shared__ unsigned long long sort_buf[];  // [pow2 >= beam_size]
  __shared__ int warp_cnt[ACC_THREADS / 32];
  __shared__ int s_accepted, s_attempted, s_invalid, s_dup, s_done;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t count = min(*count_ptr, cap);
  if (tid == 0) { s_accepted = 0; s_attempted = 0; s_invalid = 0; s_dup = 0; s_done = 0; }
  __syncthreads();
  for (int64_t base = 0; base < count; base += ACC_THREADS) {
    if (s_done) break;
    const int64_t j = base + tid;
    const uint8_t code = j < count ? accept[j] : 0;
    const bool acc = j < count && code == 2;
    const unsigned ballot = __ballot_sync(0xffffffffu, acc);
    if (lane == 0) warp_cnt[warp] = __popc(ballot);
    __syncthreads();
    int before = s_accepted;
    for (int w = 0; w < warp; ++w) before += warp_cnt[w];
    before += __popc(ballot & ((1u << lane) - 1u));
    // position of this proposal relative to the stop: the loop stops right
    // after the beam_size-th accept.
    const bool attempted = j < count && before < beam_size;
    if (acc && before < beam_size) {
      sort_buf[before] = ((unsigned long long)(uint32_t)(next_gate[j] + 0x40000000ll) << 32) |
                         (unsigned long long)(uint32_t)before;
      child_proposal[before] = j;
      // insert into the seen set
      const uint64_t key = table_key(fp[j]);
      uint64_t h = mix64(key) & (seen_capacity - 1);
      bool placed = false;
      for (int64_t probe = 0; probe < seen_capacity; ++probe, h = (h + 1) & (seen_capacity - 1)) {
        const unsigned long long prev = atomicCAS(reinterpret_cast<unsigned long long*>(&seen[h]),
                                                  EMPTY_KEY, key);
        if (prev == EMPTY_KEY || prev == key) { placed = true; break; }
      }
      if (!placed) set_status(status, GRS_ERR_WORKSPACE);
    }
    if (attempted) {
      atomicAdd(&s_attempted, 1);
      if (code == 0) atomicAdd(&s_invalid, 1);
      if (code == 1) atomicAdd(&s_dup, 1);
    }
    __syncthreads();
    if (tid == 0) {
      int tot = 0;
      for (int w = 0; w < ACC_THREADS / 32; ++w) tot += warp_cnt[w];
      s_accepted += tot;
      if (s_accepted >= beam_size) { s_accepted = beam_size; s_done = 1; }
    }
    __syncthreads();
  }
  const int n = s_accepted;
  int size = 1;
  while (size < n) size <<= 1;
  for (int i = n + tid; i < size; i += ACC_THREADS) sort_buf[i] = ~0ull;
  __syncthreads();
  for (int k2 = 2; k2 <= size; k2 <<= 1) {
    for (int jj = k2 >> 1; jj > 0; jj >>= 1) {
      for (int i = tid; i < size; i += ACC_THREADS) {
        const int l = i ^ jj;
        if (l > i) {
          const unsigned long long x = sort_buf[i], y = sort_buf[l];
          const bool asc = (i & k2) == 0;
          if (asc ? (x > y) : (x < y)) { sort_buf[i] = y; sort_buf[l] = x; }
        }
      }
      __syncthreads();
    }
  }
  // child_proposal currently holds accept order; permute by the sorted ranks.
  int64_t mine[8];
  int cnt = 0;
  for (int i = tid; i < n && cnt < 8; i += ACC_THREADS)
    mine[cnt++] = child_proposal[(uint32_t)(sort_buf[i] & 0xffffffffu)];
  __syncthreads();
  cnt = 0;
  for (int i = tid; i < n && cnt < 8; i += ACC_THREADS) child_proposal[i] = mine[cnt++];
  __syncthreads();
  if (tid == 0) {
    summary[0] = n;
    summary[1] = s_attempted;
    summary[2] = s_invalid;
    summary[3] = s_dup;
    summary[5] = n > 0 ? next_gate[child_proposal[0]] : -1;  // best child gate count
  }
}

struct MaterializeArgs {
  const int64_t* child_proposal; const int64_t* summary;
  const int64_t* rows; const int64_t* xfers; const int64_t* next_gate; const uint64_t* fp;
  const int64_t* cand_batch; const int64_t* cand_anchor; const int64_t* cand_bindings;
  int cand_pattern; const int32_t* table; const int64_t* xfer_to_source;
  int p_slots, slots;   // parent row stride; child row stride (>= every child's next slot)
  // parent state
  const int64_t* p_types; Ports p_ports; const int32_t* p_touched; const uint8_t* p_pref;
  const int32_t* p_next_slot; const int32_t* p_streak;
  // child state
  int64_t* c_types; Ports c_ports; int32_t* c_touched; uint8_t* c_pref; int32_t* c_distance;
  int32_t* c_next_slot; int32_t* c_streak; int64_t* c_gate; uint64_t* c_fp;
  // per-child action tensors for the model advance
  int64_t* a_parent; int64_t* a_xfer; int64_t* a_source; int64_t* a_src_slots; int src_pattern;
  int64_t* a_dst_slots; int64_t* a_dst_types; int dst_pattern;
  int depth;
  int32_t* status;
};

constexpr int MAT_THREADS = 256;
constexpr int MAT_MAX_CORE = 96;

__global__ void __launch_bounds__(MAT_THREADS) topology_materialize_kernel(MaterializeArgs a) {
  extern __shared__ int smem32[];
  int* dist = smem32;                   // [slots]
  int* queue = smem32 + a.slots;        // [slots]
  __shared__ int64_t s_core[MAT_MAX_CORE];
  __shared__ int s_ncore, s_head, s_tail, s_next_tail;
  __shared__ int64_t s_bind[TAB_MAXP];
  __shared__ int s_nb;
  const int i = blockIdx.x;
  if (i >= a.summary[0]) return;
  const int tid = threadIdx.x;
  const int64_t j = a.child_proposal[i];
  const int64_t row = a.rows[j];
  const int64_t x = a.xfers[j];
  const int64_t parent = a.cand_batch[row];
  const int32_t* tab = a.table + x * TAB_WIDTH;
  const int dst_len = tab[TAB_DST_LEN];
  const int64_t pb = parent * a.p_slots, cb = (int64_t)i * a.slots;
  const int32_t ns = a.p_next_slot[parent];
  if (tid == 0) {
    int nb = 0;
    for (int k = 0; k < a.cand_pattern && nb < TAB_MAXP; ++k) {
      const int64_t v = a.cand_bindings[row * a.cand_pattern + k];
      if (v >= 0) s_bind[nb++] = v;
    }
    s_nb = nb;
  }
  // 1. copy the parent rows
  for (int s = tid; s < a.slots; s += MAT_THREADS) {
    const bool has = s < a.p_slots;
    a.c_types[cb + s] = has ? a.p_types[pb + s] : -1;
    a.c_touched[cb + s] = has ? a.p_touched[pb + s] : -1;
    a.c_pref[cb + s] = 0;
    for (int p = 0; p < 4; ++p) {
      a.c_ports.out_node[(cb + s) * 4 + p] = has ? a.p_ports.out_node[(pb + s) * 4 + p] : -1;
      a.c_ports.out_port[(cb + s) * 4 + p] = has ? a.p_ports.out_port[(pb + s) * 4 + p] : -1;
      a.c_ports.in_node[(cb + s) * 4 + p] = has ? a.p_ports.in_node[(pb + s) * 4 + p] : -1;
      a.c_ports.in_port[(cb + s) * 4 + p] = has ? a.p_ports.in_port[(pb + s) * 4 + p] : -1;
    }
    dist[s] = -1;
  }
  __syncthreads();
  // 2. apply the rewrite (one thread; a handful of ports)
  if (tid == 0) {
    const int nb = s_nb;
    int ncore = 0;
    auto add_core = [&](int64_t v) {
      for (int c = 0; c < ncore; ++c) if (s_core[c] == v) return;
      if (ncore < MAT_MAX_CORE) s_core[ncore++] = v; else set_status(a.status, GRS_ERR_SHAPE);
    };
    auto is_removed = [&](int64_t v) { return in_set(s_bind, nb, v); };
    Ports cp = a.c_ports;
    // boundaries from the parent's ports (before any change)
    int64_t pred[TAB_MAXW], pred_port[TAB_MAXW], succ[TAB_MAXW], succ_port[TAB_MAXW];
    const int nw = tab[TAB_NWIRES];
    for (int w = 0; w < nw; ++w) {
      const int32_t* wr = tab + TAB_WIRES + w * 8;
      pred[w] = succ[w] = -1;
      if (wr[0] >= 0) {
        const int64_t pi = (pb + s_bind[wr[0]]) * 4 + wr[1];
        if (a.p_ports.in_node[pi] >= 0 && !is_removed(a.p_ports.in_node[pi])) {
          pred[w] = a.p_ports.in_node[pi]; pred_port[w] = a.p_ports.in_port[pi];
        }
        const int64_t si = (pb + s_bind[wr[2]]) * 4 + wr[3];
        if (a.p_ports.out_node[si] >= 0 && !is_removed(a.p_ports.out_node[si])) {
          succ[w] = a.p_ports.out_node[si]; succ_port[w] = a.p_ports.out_port[si];
        }
      }
    }
    // previous-preferred: destinations and surviving predecessors of removed slots
    for (int k = 0; k < nb; ++k) {
      for (int p = 0; p < 4; ++p) {
        const int32_t in = a.p_ports.in_node[(pb + s_bind[k]) * 4 + p];
        if (in >= 0 && !is_removed(in)) a.c_pref[cb + in] = 1;
      }
    }
    // remove every edge at a removed slot; surviving endpoints join the core
    for (int k = 0; k < nb; ++k) {
      const int64_t v = s_bind[k];
      for (int p = 0; p < 4; ++p) {
        const int64_t pi = (pb + v) * 4 + p;
        const int32_t o = a.p_ports.out_node[pi];
        if (o >= 0) {
          const int32_t op = a.p_ports.out_port[pi];
          if (!is_removed(o)) {
            cp.in_node[(cb + o) * 4 + op] = -1; cp.in_port[(cb + o) * 4 + op] = -1;
            add_core(o);
          }
        }
        const int32_t in = a.p_ports.in_node[pi];
        if (in >= 0) {
          const int32_t ip = a.p_ports.in_port[pi];
          if (!is_removed(in)) {
            cp.out_node[(cb + in) * 4 + ip] = -1; cp.out_port[(cb + in) * 4 + ip] = -1;
            add_core(in);
          }
        }
        cp.out_node[(cb + v) * 4 + p] = -1; cp.out_port[(cb + v) * 4 + p] = -1;
        cp.in_node[(cb + v) * 4 + p] = -1; cp.in_port[(cb + v) * 4 + p] = -1;
      }
      a.c_types[cb + v] = -1;
      a.c_touched[cb + v] = -1;
    }
    for (int d = 0; d < dst_len; ++d) {
      a.c_types[cb + ns + d] = tab[TAB_DST_TYPES + d];
      a.c_pref[cb + ns + d] = 1;
      add_core(ns + d);
    }
    auto add_edge = [&](int64_t s, int64_t d, int64_t sp, int64_t dp) {
      cp.out_node[(cb + s) * 4 + sp] = (int32_t)d; cp.out_port[(cb + s) * 4 + sp] = (int32_t)dp;
      cp.in_node[(cb + d) * 4 + dp] = (int32_t)s; cp.in_port[(cb + d) * 4 + dp] = (int32_t)sp;
      add_core(s);
      add_core(d);
    };
    for (int w = 0; w < nw; ++w) {
      const int32_t* wr = tab + TAB_WIRES + w * 8;
      if (wr[4] >= 0) {
        if (pred[w] >= 0) add_edge(pred[w], ns + wr[4], pred_port[w], wr[5]);
        if (succ[w] >= 0) add_edge(ns + wr[6], succ[w], wr[7], succ_port[w]);
      } else if (pred[w] >= 0 && succ[w] >= 0) {
        add_edge(pred[w], succ[w], pred_port[w], succ_port[w]);
      }
    }
    const int nint = tab[TAB_NINT];
    for (int e = 0; e < nint; ++e) {
      const int32_t* ie = tab + TAB_INT + e * 4;
      add_edge(ns + ie[0], ns + ie[1], ie[2], ie[3]);
    }
    for (int c = 0; c < ncore; ++c) {
      a.c_touched[cb + s_core[c]] = a.depth;
      dist[s_core[c]] = 0;
      queue[c] = (int)s_core[c];
    }
    s_ncore = ncore;
    s_head = 0;
    s_tail = ncore;
    s_next_tail = ncore;
    // scalars and the action tensors of this child
    const int64_t anchor = a.cand_anchor[row];
    a.c_streak[i] = a.p_pref[pb + anchor] ? a.p_streak[parent] + 1 : 0;
    a.c_next_slot[i] = ns + dst_len;
    a.c_gate[i] = a.next_gate[j];
    a.c_fp[i] = a.fp[j];
    a.a_parent[i] = parent;
    a.a_xfer[i] = x;
    a.a_source[i] = a.xfer_to_source[x];
    for (int k = 0; k < a.src_pattern; ++k) a.a_src_slots[(int64_t)i * a.src_pattern + k] = k < nb ? s_bind[k] : -1;
    for (int d = 0; d < a.dst_pattern; ++d) {
      a.a_dst_slots[(int64_t)i * a.dst_pattern + d] = d < dst_len ? ns + d : -1;
      a.a_dst_types[(int64_t)i * a.dst_pattern + d] = d < dst_len ? tab[TAB_DST_TYPES + d] : -1;
    }
  }
  __syncthreads();
  // 3. level-synchronous BFS from the core over the child graph
  int level = 0;
  while (true) {
    const int head = s_head, tail = s_tail;
    if (head >= tail) break;
    for (int q = head + tid; q < tail; q += MAT_THREADS) {
      const int64_t v = queue[q];
      for (int p = 0; p < 8; ++p) {
        const int32_t nb = p < 4 ? a.c_ports.out_node[(cb + v) * 4 + p]
                                 : a.c_ports.in_node[(cb + v) * 4 + (p - 4)];
        if (nb >= 0 && nb < a.slots && atomicCAS(&dist[nb], -1, level + 1) == -1) {
          const int slot = atomicAdd(&s_next_tail, 1);
          if (slot < a.slots) queue[slot] = nb;
        }
      }
    }
    __syncthreads();
    if (tid == 0) { s_head = tail; s_tail = min(s_next_tail, a.slots); }
    ++level;
    __syncthreads();
  }
  for (int s = tid; s < a.slots; s += MAT_THREADS) {
    const bool live = a.c_types[cb + s] >= 0;
    const int d = dist[s];
    a.c_distance[cb + s] = live ? (d >= 0 ? min(d, 4) : 5) : 5;
  }
}

// Initial topology of beam rows from port arrays already filled: fingerprint
// and scalars (one CTA per beam; block reduce of the XOR components).
__global__ void topology_fingerprint_kernel(const int64_t* types, Ports ports, int slots,
                                            uint64_t* fp) {
  __shared__ unsigned long long part[256];
  const int b = blockIdx.x;
  unsigned long long acc = 0;
  for (int s = threadIdx.x; s < slots; s += blockDim.x) {
    const int64_t t = types[(int64_t)b * slots + s];
    if (t >= 0) acc ^= node_component(s, t);
    for (int p = 0; p < 4; ++p) {
      const int64_t pi = ((int64_t)b * slots + s) * 4 + p;
      if (ports.out_node[pi] >= 0) acc ^= edge_component(s, ports.out_node[pi], p, ports.out_port[pi]);
    }
  }
  part[threadIdx.x] = acc;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) part[threadIdx.x] ^= part[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) fp[b] = part[0];
}

}  // namespace grs

using namespace grs;

__global__ void topology_extent_kernel(const int64_t* child_proposal, const int64_t* summary,
                                       const int64_t* rows, const int64_t* xfers,
                                       const int64_t* cand_batch, const int32_t* table,
                                       const int32_t* next_slot, int64_t* out_max) {
  __shared__ int best;
  if (threadIdx.x == 0) best = 0;
  __syncthreads();
  const int n = (int)summary[0];
  int local = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t j = child_proposal[i];
    const int64_t row = rows[j];
    const int v = next_slot[cand_batch[row]] + table[xfers[j] * TAB_WIDTH + TAB_DST_LEN];
    local = max(local, v);
  }
  atomicMax(&best, local);
  __syncthreads();
  if (threadIdx.x == 0) *out_max = best;
}

extern "C" int grs_topology_table_width(void) { return TAB_WIDTH; }

extern "C" int grs_topology_plan(int64_t count_cap, const int64_t* count, const int64_t* rows,
                                 const int64_t* xfers, const int64_t* next_gate,
                                 const int64_t* cand_batch, const int64_t* cand_bindings,
                                 int cand_pattern, const int32_t* table, const int64_t* types,
                                 int32_t* out_node, int32_t* out_port, int32_t* in_node,
                                 int32_t* in_port, int slots, const int32_t* next_slot,
                                 const uint64_t* fingerprint, uint8_t* valid, uint64_t* fp_out,
                                 int32_t* status, void* stream) {
  if (count_cap <= 0) return GRS_OK;
  PlanArgs a{count_cap, count, rows, xfers, next_gate, cand_batch, cand_bindings, cand_pattern,
             table, types, Ports{out_node, out_port, in_node, in_port}, slots, next_slot,
             fingerprint, valid, fp_out, status};
  topology_plan_kernel<<<ceil_div(count_cap, 128), 128, 0, grs::counted((cudaStream_t)stream)>>>(a);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_topology_accept(int64_t count_cap, const int64_t* count, const uint8_t* valid,
                                   const uint64_t* fp, const int64_t* next_gate, int beam_size,
                                   uint64_t* step_keys, int32_t* step_first,
                                   int64_t step_capacity, uint64_t* seen, int64_t seen_capacity,
                                   uint8_t* classes, int64_t* child_proposal, int64_t* summary,
                                   const int64_t* rows, const int64_t* xfers,
                                   const int64_t* cand_batch, const int32_t* table,
                                   const int32_t* next_slot, int32_t* status, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (count_cap <= 0 || beam_size <= 0 || beam_size > 8192) return GRS_ERR_SHAPE;
  if ((step_capacity & (step_capacity - 1)) || (seen_capacity & (seen_capacity - 1)))
    return GRS_ERR_SHAPE;
  int size = 1;
  while (size < beam_size) size <<= 1;
  const size_t smem = (size_t)size * sizeof(unsigned long long);
  if (smem > 200 * 1024) return GRS_ERR_SHAPE;
  cudaMemsetAsync(step_keys, 0, step_capacity * sizeof(uint64_t), s);
  cudaMemsetAsync(step_first, 0x7f, step_capacity * sizeof(int32_t), s);
  topology_first_kernel<<<ceil_div(count_cap, 256), 256, 0, grs::counted(s)>>>(valid, fp, count_cap, step_keys,
                                                                step_first, step_capacity, status);
  topology_classify_kernel<<<ceil_div(count_cap, 256), 256, 0, grs::counted(s)>>>(
      valid, fp, count_cap, step_keys, step_first, step_capacity, seen, seen_capacity, classes);
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(topology_accept_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         200 * 1024);
    attr[dev] = true;
  }
  topology_accept_kernel<<<1, ACC_THREADS, smem, grs::counted(s)>>>(classes, count, count_cap, fp, next_gate,
                                                      beam_size, seen, seen_capacity,
                                                      child_proposal, summary, status);
  if (rows != nullptr)
    topology_extent_kernel<<<1, 256, 0, grs::counted(s)>>>(child_proposal, summary, rows, xfers,
                                                           cand_batch, table, next_slot,
                                                           summary + 4);
  else
    cudaMemsetAsync(summary + 4, 0, sizeof(int64_t), s);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_topology_seen_insert(const uint64_t* fp, int64_t n, uint64_t* seen,
                                        int64_t seen_capacity, int32_t* status, void* stream);

extern "C" int grs_topology_materialize(
    int max_children, const int64_t* child_proposal, const int64_t* summary, const int64_t* rows,
    const int64_t* xfers, const int64_t* next_gate, const uint64_t* fp, const int64_t* cand_batch,
    const int64_t* cand_anchor, const int64_t* cand_bindings, int cand_pattern,
    const int32_t* table, const int64_t* xfer_to_source, int p_slots, int slots,
    const int64_t* p_types,
    const int32_t* p_out_node, const int32_t* p_out_port, const int32_t* p_in_node,
    const int32_t* p_in_port, const int32_t* p_touched, const uint8_t* p_pref,
    const int32_t* p_next_slot, const int32_t* p_streak, int64_t* c_types, int32_t* c_out_node,
    int32_t* c_out_port, int32_t* c_in_node, int32_t* c_in_port, int32_t* c_touched,
    uint8_t* c_pref, int32_t* c_distance, int32_t* c_next_slot, int32_t* c_streak,
    int64_t* c_gate, uint64_t* c_fp, int64_t* a_parent, int64_t* a_xfer, int64_t* a_source,
    int64_t* a_src_slots, int src_pattern, int64_t* a_dst_slots, int64_t* a_dst_types,
    int dst_pattern, int depth, int32_t* status, void* stream) {
  if (max_children <= 0) return GRS_OK;
  if (slots <= 0 || slots > 12000 || p_slots <= 0 || p_slots > slots) return GRS_ERR_SHAPE;
  MaterializeArgs a{child_proposal, summary, rows, xfers, next_gate, fp, cand_batch, cand_anchor,
                    cand_bindings, cand_pattern, table, xfer_to_source, p_slots, slots, p_types,
                    Ports{const_cast<int32_t*>(p_out_node), const_cast<int32_t*>(p_out_port),
                          const_cast<int32_t*>(p_in_node), const_cast<int32_t*>(p_in_port)},
                    p_touched, p_pref, p_next_slot, p_streak, c_types,
                    Ports{c_out_node, c_out_port, c_in_node, c_in_port}, c_touched, c_pref,
                    c_distance, c_next_slot, c_streak, c_gate, c_fp, a_parent, a_xfer, a_source,
                    a_src_slots, src_pattern, a_dst_slots, a_dst_types, dst_pattern, depth,
                    status};
  const size_t smem = (size_t)2 * slots * sizeof(int);
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(topology_materialize_kernel,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
    attr[dev] = true;
  }
  topology_materialize_kernel<<<max_children, MAT_THREADS, smem, grs::counted((cudaStream_t)stream)>>>(a);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

extern "C" int grs_topology_fingerprint(const int64_t* types, const int32_t* out_node,
                                        const int32_t* out_port, const int32_t* in_node,
                                        const int32_t* in_port, int batch, int slots,
                                        uint64_t* fp, void* stream) {
  if (batch <= 0) return GRS_OK;
  topology_fingerprint_kernel<<<batch, 256, 0, grs::counted((cudaStream_t)stream)>>>(
      types, Ports{const_cast<int32_t*>(out_node), const_cast<int32_t*>(out_port),
                   const_cast<int32_t*>(in_node), const_cast<int32_t*>(in_port)},
      slots, fp);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}

__global__ void seen_insert_kernel(const uint64_t* fp, int64_t n, uint64_t* seen, int64_t cap,
                                   int32_t* status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t key = table_key(fp[i]);
  uint64_t h = mix64(key) & (cap - 1);
  for (int64_t probe = 0; probe < cap; ++probe, h = (h + 1) & (cap - 1)) {
    const unsigned long long prev =
        atomicCAS(reinterpret_cast<unsigned long long*>(&seen[h]), EMPTY_KEY, key);
    if (prev == EMPTY_KEY || prev == key) return;
  }
  set_status(status, GRS_ERR_WORKSPACE);
}

extern "C" int grs_topology_seen_insert(const uint64_t* fp, int64_t n, uint64_t* seen,
                                        int64_t seen_capacity, int32_t* status, void* stream) {
  if (n <= 0) return GRS_OK;
  if (seen_capacity & (seen_capacity - 1)) return GRS_ERR_SHAPE;
  seen_insert_kernel<<<ceil_div(n, 256), 256, 0, grs::counted((cudaStream_t)stream)>>>(fp, n, seen,
                                                                         seen_capacity, status);
  GRS_CUDA_CHECK_LAUNCH();
  return GRS_OK;
}
