// Routed mixture-of-experts for the verify block (reference/fused_ops.py:148-173,
// fused/model.py:296-307, fused/quantization.py:181-202).
//
//  route   one warp per token: fp32 softmax of the router logits, top-k selection that
//          reproduces torch.topk's CPU order exactly (below), renormalized weights cast
//          to the activation dtype; then one CTA-wide pass builds, per active expert in
//          ascending id, the list of (token, slot) pairs routed to it.
//  up      CTA = (expert slot, 16-wide intermediate tile): gate and up rows streamed once,
//          K split over 8 warps, SiLU(gate) * up in the reference's rounding order.
//  down    CTA = (expert slot, 128 output rows): each pair's raw fp32 expert output goes
//          to its own (token, slot) row, so the combine (ascending expert order, bf16
//          rounding at each add as the reference) is deterministic.
//  Slot 0 is the shared expert (all tokens), slots 1.. the active routed experts.
//
// torch.topk order.  The reference selects with torch.topk on CPU
// (reference/fused_ops.py:163).  ATen copies (value, index) pairs into a queue in index
// order and, when k*64 > n, runs std::nth_element(k-1) then std::sort of the first k-1
// entries (GNU libstdc++ introselect: median-of-3 pivot moved to the front, unguarded
// Hoare partition, insertion sort below 4 elements, heap select past 2*log2(n) levels),
// else std::partial_sort (heap select + sort heap); comparator a.value > b.value.  Ties
// therefore resolve by the partition history, not by index.  Each partition is run
// here in parallel across the warp in closed form: the i-th left stop (value <= pivot,
// ascending) swaps with the i-th right stop (value >= pivot, descending) while the
// first is left of the second; the cut is the next left stop, or the last right stop
// swapped, whichever comes first.  The sequential steps (pivot choice, small sorts,
// heap fallback) run on lane 0.  Values compared are the bf16 router logits, which
// order exactly as torch's fp32 probabilities (exp is monotone; equal logits give
// equal probabilities).
#include <cooperative_groups.h>
#include <atomic>
#include <cstring>
#include <mutex>

#include "bulk_ring.cuh"
#include "stream_gemm.cuh"
#include "umma.cuh"

namespace qw {

namespace cg = cooperative_groups;

// ------------------------------------------------------------------ route workspace
struct RouteView {
  int32_t* topk_idx;    // [T*k]
  float* topk_w;        // [T*k]  (value of the activation dtype)
  float* shared_gate;   // [T]
  int32_t* n_active;    // [4]: [0] active experts, [1..3] unused
  int32_t* active;      // [min(E, T*k)]
  int32_t* pair_off;    // [min(E, T*k) + 1]
  int32_t* pair_tok;    // [T*k]
  int32_t* pair_slot;   // [T*k]
};

__host__ __device__ inline int64_t route_ints(int T, int E, int k) {
  const int64_t na = (E < T * k) ? E : T * k;
  return 2LL * T * k + T + 4 + na + na + 1 + 2LL * T * k;
}

__host__ __device__ inline RouteView route_view(void* ws, int T, int E, int k) {
  RouteView v;
  const int64_t na = (E < T * k) ? E : T * k;
  int32_t* p = static_cast<int32_t*>(ws);
  v.topk_idx = p; p += T * k;
  v.topk_w = reinterpret_cast<float*>(p); p += T * k;
  v.shared_gate = reinterpret_cast<float*>(p); p += T;
  v.n_active = p; p += 4;
  v.active = p; p += na;
  v.pair_off = p; p += na + 1;
  v.pair_tok = p; p += T * k;
  v.pair_slot = p;
  return v;
}

// Staged gate/up input of a routed block, right after the routing ints: a 256-byte
// header (the x pointer and a shape key it was staged for), x16 [T, H] (the bf16
// activations as fp16, saturated) and xsum [T, H / G] (group_xsum_f16 of each token's
// K groups; room for G >= 32).  qw_moe_route_x writes it once per block so that the
// gate/up kernel's CTAs need not each convert and sum x.
__host__ __device__ inline int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }
__host__ __device__ inline int64_t stage_off(int T, int E, int k) { return align256(route_ints(T, E, k) * 4); }
__host__ __device__ inline int64_t stage_bytes(int T, int H) {
  return 256 + align256(static_cast<int64_t>(T) * H * 2) + align256(static_cast<int64_t>(T) * (H / 32) * 4);
}
__host__ __device__ inline unsigned long long stage_key(int T, int H, int G) {
  return (static_cast<unsigned long long>(T) << 40) | (static_cast<unsigned long long>(H) << 8) |
         static_cast<unsigned long long>(G);
}
struct StageView {
  unsigned long long* tag;   // [0] x pointer (0: nothing staged), [1] stage_key
  __half* x16;
  float* xsum;
};
__host__ __device__ inline StageView stage_view(void* ws, int T, int E, int k, int H) {
  uint8_t* p = static_cast<uint8_t*>(ws) + stage_off(T, E, k);
  StageView v;
  v.tag = reinterpret_cast<unsigned long long*>(p);
  v.x16 = reinterpret_cast<__half*>(p + 256);
  v.xsum = reinterpret_cast<float*>(p + 256 + align256(static_cast<int64_t>(T) * H * 2));
  return v;
}

// ------------------------------------------------------------------ libstdc++ emulation
struct Q {
  float* v;
  int32_t* i;
  __device__ __forceinline__ bool gt(int a, int b) const { return v[a] > v[b]; }
  __device__ __forceinline__ void swap(int a, int b) const {
    float tv = v[a]; v[a] = v[b]; v[b] = tv;
    int32_t ti = i[a]; i[a] = i[b]; i[b] = ti;
  }
};

// libstdc++ __move_median_to_first under a > b: every lane makes the choice from one
// parallel read of the three values, lane 0 swaps (the warp synchronizes after).
__device__ __forceinline__ void warp_move_median_to_first(const Q& q, int result, int a, int b, int c, int lane) {
  const float va = q.v[a], vb = q.v[b], vc = q.v[c];
  int m;
  if (va > vb) m = vb > vc ? b : (va > vc ? c : a);
  else m = va > vc ? a : (vb > vc ? c : b);
  if (lane == 0) q.swap(result, m);
}

__device__ void q_insertion_sort(const Q& q, int first, int last) {
  for (int i = first + 1; i < last; ++i) {
    const float vv = q.v[i];
    const int32_t vi = q.i[i];
    if (vv > q.v[first]) {
      for (int j = i; j > first; --j) { q.v[j] = q.v[j - 1]; q.i[j] = q.i[j - 1]; }
      q.v[first] = vv; q.i[first] = vi;
    } else {
      int hole = i, prev = i - 1;
      while (vv > q.v[prev]) { q.v[hole] = q.v[prev]; q.i[hole] = q.i[prev]; hole = prev; --prev; }
      q.v[hole] = vv; q.i[hole] = vi;
    }
  }
}

__device__ void q_push_heap(const Q& q, int first, int hole, int top, float vv, int32_t vi) {
  int parent = (hole - 1) / 2;
  while (hole > top && q.v[first + parent] > vv) {
    q.v[first + hole] = q.v[first + parent]; q.i[first + hole] = q.i[first + parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  q.v[first + hole] = vv; q.i[first + hole] = vi;
}

__device__ void q_adjust_heap(const Q& q, int first, int hole, int len, float vv, int32_t vi) {
  const int top = hole;
  int child = hole;
  while (child < (len - 1) / 2) {
    child = 2 * (child + 1);
    if (q.v[first + child] > q.v[first + child - 1]) --child;
    q.v[first + hole] = q.v[first + child]; q.i[first + hole] = q.i[first + child];
    hole = child;
  }
  if ((len & 1) == 0 && child == (len - 2) / 2) {
    child = 2 * (child + 1);
    q.v[first + hole] = q.v[first + child - 1]; q.i[first + hole] = q.i[first + child - 1];
    hole = child - 1;
  }
  q_push_heap(q, first, hole, top, vv, vi);
}

__device__ void q_make_heap(const Q& q, int first, int last) {
  const int len = last - first;
  if (len < 2) return;
  int parent = (len - 2) / 2;
  while (true) {
    q_adjust_heap(q, first, parent, len, q.v[first + parent], q.i[first + parent]);
    if (parent == 0) return;
    --parent;
  }
}

__device__ void q_heap_select(const Q& q, int first, int middle, int last) {
  q_make_heap(q, first, middle);
  for (int i = middle; i < last; ++i) {
    if (q.v[i] > q.v[first]) {
      const float vv = q.v[i];
      const int32_t vi = q.i[i];
      q.v[i] = q.v[first]; q.i[i] = q.i[first];
      q_adjust_heap(q, first, 0, middle - first, vv, vi);
    }
  }
}

// Parallel unguarded Hoare partition of [a, b) around the pivot at a-1; returns the cut.
// pos_l / pos_r: per-warp scratch of >= (b - a + 1) entries.
__device__ int warp_partition(const Q& q, int a, int b, int16_t* pos_l, int16_t* pos_r, int lane) {
  const float p = q.v[a - 1];
  int nl = 0, nr = 0;
  // left stops ascending over [a, b)
  for (int base = a; base < b; base += 32) {
    const int i = base + lane;
    const bool is_l = i < b && !(q.v[i] > p);
    const unsigned m = __ballot_sync(0xffffffffu, is_l);
    if (is_l) pos_l[nl + __popc(m & ((1u << lane) - 1))] = static_cast<int16_t>(i);
    nl += __popc(m);
  }
  // right stops descending over [a-1, b)
  for (int top = b - 1; top >= a - 1; top -= 32) {
    const int j = top - lane;
    const bool is_r = j >= a - 1 && !(p > q.v[j]);
    const unsigned m = __ballot_sync(0xffffffffu, is_r);
    if (is_r) pos_r[nr + __popc(m & ((1u << lane) - 1))] = static_cast<int16_t>(j);
    nr += __popc(m);
  }
  __syncwarp();
  // pairs m with L[m] < R[m] form a prefix
  int mstar = 0;
  const int lim = nl < nr ? nl : nr;
  for (int base = 0; base < lim; base += 32) {
    const int m = base + lane;
    const bool ok = m < lim && pos_l[m] < pos_r[m];
    const unsigned bal = __ballot_sync(0xffffffffu, ok);
    mstar += __popc(bal);
    if (bal != 0xffffffffu) break;
  }
  for (int m = lane; m < mstar; m += 32) q.swap(pos_l[m], pos_r[m]);
  __syncwarp();
  if (mstar == 0) return pos_l[0];
  const int lm = mstar < nl ? pos_l[mstar] : 1 << 30;
  const int rm = pos_r[mstar - 1];
  return lm < rm ? lm : rm;
}

// The same partition for ranges of at most 32 IT elements (b - (a - 1) <= 32 IT; IT = 9
// covers every router of <= 256 experts): all ballots first, then the stop positions
// from prefix counts, then the pair scan unrolled, so no loop carries a memory
// dependency.
template <int IT>
__device__ int warp_partition_small(const Q& q, int a, int b, int16_t* pos_l, int16_t* pos_r, int lane) {
  const float p = q.v[a - 1];
  const unsigned lt = (1u << lane) - 1u;
  const int itn = (b - a + 32) / 32;   // 32-wide passes over [a - 1, b)
  // every value load first, indices clamped into [a - 1, b) and the out-of-range lanes
  // masked in the ballots: one shared-memory round trip instead of one per pass
  float vl[IT], vr[IT];
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    vl[it] = q.v[min(a + 32 * it + lane, b - 1)];
    vr[it] = q.v[max(b - 1 - 32 * it - lane, a - 1)];
  }
  unsigned mL[IT], mR[IT];
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    mL[it] = __ballot_sync(0xffffffffu, it < itn && a + 32 * it + lane < b && !(vl[it] > p));
    mR[it] = __ballot_sync(0xffffffffu, it < itn && b - 1 - 32 * it - lane >= a - 1 && !(p > vr[it]));
  }
  int nl = 0, nr = 0;
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    if ((mL[it] >> lane) & 1u) pos_l[nl + __popc(mL[it] & lt)] = static_cast<int16_t>(a + 32 * it + lane);
    nl += __popc(mL[it]);
    if ((mR[it] >> lane) & 1u) pos_r[nr + __popc(mR[it] & lt)] = static_cast<int16_t>(b - 1 - 32 * it - lane);
    nr += __popc(mR[it]);
  }
  __syncwarp();
  // pairs m with L[m] < R[m] form a prefix: its length is the first failing m (the stop
  // lists are read once, every pass at once, and kept for the swaps)
  const int lim = nl < nr ? nl : nr;
  const int mcap = lim > 0 ? lim - 1 : 0;
  int pl[IT], pr[IT];
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int m = min(32 * it + lane, mcap);
    pl[it] = pos_l[m];
    pr[it] = pos_r[m];
  }
  int mstar = lim;
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int m = 32 * it + lane;
    const unsigned bad = __ballot_sync(0xffffffffu, m < lim && !(pl[it] < pr[it]));
    if (bad && mstar == lim && 32 * it < lim) mstar = 32 * it + __ffs(bad) - 1;
  }
#pragma unroll
  for (int it = 0; it < IT; ++it)
    if (32 * it + lane < mstar) q.swap(pl[it], pr[it]);
  __syncwarp();
  if (mstar == 0) return pos_l[0];
  const int lm = mstar < nl ? pos_l[mstar] : 1 << 30;
  const int rm = pos_r[mstar - 1];
  return lm < rm ? lm : rm;
}

// The introselect loop below once [first, last) has at most 32 NR elements: the range is
// held NR elements per lane (register j of lane l = position first + 32 j + l at entry)
// and each step runs in registers.  The median of three comes from shuffled values; the
// partition's left stops (ascending) and right stops (descending) come from ballots, the
// m-th left stop is paired with the m-th right stop through two rank tables, the pairs
// with L[m] < R[m] (a prefix) swap by shuffles, and the cut is the sequential
// algorithm's.  Every step makes the same exchanges as the shared-memory code, so the
// arrangement is the same; the range goes back to q at exit, with first / last / depth
// advanced.  Stops when the range is <= 3 or depth reaches 0.  Registers are only ever
// selected by warp-uniform or unrolled indices.
template <int NR>
__device__ void warp_introselect_regs(const Q& q, int& first, int& last, int nth, int& depth, int16_t* slot_l,
                                      int16_t* slot_r, int lane) {
  const int base = first, wlen = last - first;
  const unsigned lt = (1u << lane) - 1u, gt = ~((2u << lane) - 1u);
  float rv[NR];
  int32_t ri[NR];
#pragma unroll
  for (int j = 0; j < NR; ++j) {
    const int o = 32 * j + lane;
    rv[j] = o < wlen ? q.v[base + o] : 0.f;
    ri[j] = o < wlen ? q.i[base + o] : 0;
  }
  // value / index at the warp-uniform offset o of the range
  auto v_at = [&](int o) {
    float x = rv[0];
#pragma unroll
    for (int j = 1; j < NR; ++j) x = (o >> 5) == j ? rv[j] : x;
    return __shfl_sync(0xffffffffu, x, o & 31);
  };
  auto i_at = [&](int o) {
    int32_t x = ri[0];
#pragma unroll
    for (int j = 1; j < NR; ++j) x = (o >> 5) == j ? ri[j] : x;
    return __shfl_sync(0xffffffffu, x, o & 31);
  };
  while (last - first > 3 && depth > 0) {
    --depth;
    // __move_median_to_first(first, first + 1, mid, last - 1)
    const int mid = first + (last - first) / 2;
    const float va = v_at(first + 1 - base), vb = v_at(mid - base), vc = v_at(last - 1 - base);
    int m;
    if (va > vb) m = vb > vc ? mid : (va > vc ? last - 1 : first + 1);
    else m = va > vc ? first + 1 : (vb > vc ? last - 1 : mid);
    if (m != first) {
      const int rf = first - base, rm = m - base;
      const float vf = v_at(rf), vm = v_at(rm);
      const int32_t jf = i_at(rf), jm = i_at(rm);
#pragma unroll
      for (int j = 0; j < NR; ++j) {
        const int o = 32 * j + lane;
        if (o == rf) { rv[j] = vm; ri[j] = jm; }
        if (o == rm) { rv[j] = vf; ri[j] = jf; }
      }
    }
    // unguarded partition of [a, b) = [first + 1, last) around the pivot at first
    const int a = first + 1, b = last;
    const float p = v_at(first - base);
    bool is_l[NR], is_r[NR];
    int rl[NR], rr[NR];
    unsigned ml[NR], mr[NR];
    int nl = 0, nr = 0;
#pragma unroll
    for (int j = 0; j < NR; ++j) {
      const int pos = base + 32 * j + lane;
      is_l[j] = pos >= a && pos < b && !(rv[j] > p);
      is_r[j] = pos >= a - 1 && pos < b && !(p > rv[j]);
      ml[j] = __ballot_sync(0xffffffffu, is_l[j]);
      mr[j] = __ballot_sync(0xffffffffu, is_r[j]);
      rl[j] = nl + __popc(ml[j] & lt);   // rank among the left stops, ascending
      nl += __popc(ml[j]);
      nr += __popc(mr[j]);
    }
    int above = 0;   // right stops in registers after j
#pragma unroll
    for (int j = NR - 1; j >= 0; --j) {
      rr[j] = above + __popc(mr[j] & gt);   // rank among the right stops, descending
      above += __popc(mr[j]);
    }
#pragma unroll
    for (int j = 0; j < NR; ++j) {
      if (is_l[j]) slot_l[rl[j]] = static_cast<int16_t>(32 * j + lane);
      if (is_r[j]) slot_r[rr[j]] = static_cast<int16_t>(32 * j + lane);
    }
    __syncwarp();
    int mstar = 0;
#pragma unroll
    for (int j = 0; j < NR; ++j)
      mstar += __popc(__ballot_sync(0xffffffffu, is_l[j] && rl[j] < nr && 32 * j + lane < slot_r[rl[j]]));
    int src[NR];
#pragma unroll
    for (int j = 0; j < NR; ++j) {
      src[j] = 32 * j + lane;
      if (is_l[j] && rl[j] < mstar) src[j] = slot_r[rl[j]];
      if (is_r[j] && rr[j] < mstar) src[j] = slot_l[rr[j]];
    }
    int cut;
    if (mstar == 0) {
      cut = base + slot_l[0];
    } else {
      const int lm = mstar < nl ? base + slot_l[mstar] : 1 << 30;
      const int rm2 = base + slot_r[mstar - 1];
      cut = lm < rm2 ? lm : rm2;
    }
    __syncwarp();   // the tables are rewritten by the next step
    float nv[NR];
    int32_t ni[NR];
#pragma unroll
    for (int j = 0; j < NR; ++j) {
      nv[j] = 0.f;
      ni[j] = 0;
#pragma unroll
      for (int jj = 0; jj < NR; ++jj) {
        const float tv = __shfl_sync(0xffffffffu, rv[jj], src[j] & 31);
        const int32_t ti = __shfl_sync(0xffffffffu, ri[jj], src[j] & 31);
        if ((src[j] >> 5) == jj) { nv[j] = tv; ni[j] = ti; }
      }
    }
#pragma unroll
    for (int j = 0; j < NR; ++j) { rv[j] = nv[j]; ri[j] = ni[j]; }
    if (cut <= nth) first = cut;
    else last = cut;
  }
#pragma unroll
  for (int j = 0; j < NR; ++j) {
    const int o = 32 * j + lane;
    if (o < wlen) { q.v[base + o] = rv[j]; q.i[base + o] = ri[j]; }
  }
  __syncwarp();
}

// libstdc++ __insertion_sort of [first, first + n) under a > b, n <= 32, in parallel: it
// is a stable descending sort, so element i goes to the number of elements greater than
// it plus the number of equal ones before it.
__device__ void warp_stable_sort_desc(const Q& q, int first, int n, int lane) {
  float vi = 0.f;
  int32_t ii = 0;
  int rank = 0;
  if (lane < n) {
    vi = q.v[first + lane];
    ii = q.i[first + lane];
    for (int j = 0; j < n; ++j) {
      const float vj = q.v[first + j];
      rank += (vj > vi) || (j < lane && !(vj > vi) && !(vi > vj));
    }
  }
  __syncwarp();
  if (lane < n) { q.v[first + rank] = vi; q.i[first + rank] = ii; }
  __syncwarp();
}

// torch.topk(values, k) order for one row held in q.v / q.i (initialized in index order).
// Leaves the selected pairs in q[0..k).
__device__ void warp_topk(const Q& q, int n, int k, int16_t* pos_l, int16_t* pos_r, int lane) {
  if (k * 64 <= n) {  // std::partial_sort
    if (lane == 0) {
      q_heap_select(q, 0, k, n);
      for (int last = k; last > 1;) {
        --last;
        const float vv = q.v[last];
        const int32_t vi = q.i[last];
        q.v[last] = q.v[0]; q.i[last] = q.i[0];
        q_adjust_heap(q, 0, 0, last, vv, vi);
      }
    }
    __syncwarp();
    return;
  }
  int first = 0, last = n;
  const int nth = k - 1;
  int depth = 2 * (31 - __clz(n));
  bool heap_done = false;
  while (last - first > 3) {
    if (depth == 0) {
      if (lane == 0) {
        q_heap_select(q, first, nth + 1, last);
        q.swap(first, nth);
      }
      heap_done = true;
      break;
    }
    if (last - first <= 64) {   // the rest of the loop in registers (same steps)
      if (last - first <= 32) warp_introselect_regs<1>(q, first, last, nth, depth, pos_l, pos_r, lane);
      else warp_introselect_regs<2>(q, first, last, nth, depth, pos_l, pos_r, lane);
      continue;
    }
    --depth;
    const int mid = first + (last - first) / 2;
    warp_move_median_to_first(q, first, first + 1, mid, last - 1, lane);
    __syncwarp();
    const int cut = last - first <= 160   ? warp_partition_small<5>(q, first + 1, last, pos_l, pos_r, lane)
                    : last - first <= 288 ? warp_partition_small<9>(q, first + 1, last, pos_l, pos_r, lane)
                                          : warp_partition(q, first + 1, last, pos_l, pos_r, lane);
    if (cut <= nth) first = cut;
    else last = cut;
  }
  if (!heap_done) warp_stable_sort_desc(q, first, last - first, lane);
  if (k - 1 <= 32) {
    warp_stable_sort_desc(q, 0, k - 1, lane);
  } else {
    if (lane == 0) q_insertion_sort(q, 0, k - 1);
    __syncwarp();
  }
}

// ------------------------------------------------------------------ route kernels
// route_topk_kernel: one warp (CTA) per token.
//
// Selection.  When the k+1 largest logits of a row are strictly ordered
// (v0 > v1 > ... > v_{k-1} > v_k), every correct top-k returns the same indices in the
// same (descending) order, torch.topk's included, so the warp extracts them directly
// from registers (k+1 rounds of a warp arg-max).  A row with any tie among them (or
// more than 256 experts) runs the libstdc++ emulation above, which reproduces the order
// torch.topk gives tied values.  Dynamic smem (emulation rows): E floats + E ints +
// 2 * (E + 2) int16.
constexpr int ROUTE_MAXJ = 8;  // logits per lane on the fast path (E <= 256)

// One token's row of x -> x16 and its group sums (warp, lanes = 8-element segments).
// The row's loads are all issued before the first is used (8 per lane for H = 2048), so
// the staging costs one load latency, not one per 256 columns.
template <int G>
__device__ __forceinline__ void stage_row(const __nv_bfloat16* xr, __half* dst, float* xs, int H, int lane) {
  constexpr int NB = 8;
  for (int b0 = 0; b0 < H / 256; b0 += NB) {
    uint4 raw[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b)
      if (b0 + b < H / 256) raw[b] = __ldg(reinterpret_cast<const uint4*>(xr + ((b0 + b) * 32 + lane) * 8));
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (b0 + b < H / 256) {
        const int seg = (b0 + b) * 32 + lane;
        const uint4 v = bf16x8_to_f16x8(raw[b]);
        *reinterpret_cast<uint4*>(dst + seg * 8) = v;
        const float xg = warp_group_xsum_f16<G>(sum8_f16(v), lane);
        if (lane % (G / 8) == 0) xs[seg * 8 / G] = xg;
      }
    }
  }
}

// ROUTE_TPB tokens per CTA (one warp each): few CTAs, so they fit beside the router
// GEMV's clusters and stage x while it still runs.
constexpr int ROUTE_TPB = 4;

__host__ __device__ inline size_t route_warp_smem(int E) { return ((E * 8 + 2 * (E + 2) * 2) + 15) / 16 * 16; }

template <typename LT>
__global__ void __launch_bounds__(32 * ROUTE_TPB) route_topk_kernel(const LT* __restrict__ logits, int64_t ldl,
                                                                   int T, int E, int k, int shared_col,
                                                                   int act_is_f16, void* ws,
                                                                   const __nv_bfloat16* __restrict__ x, int H,
                                                                   int G, int tie_order) {
  extern __shared__ __align__(16) uint8_t smem_all[];
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * ROUTE_TPB + (threadIdx.x >> 5);   // this warp's token
  if (t >= T) return;   // (another warp of the CTA waits for the predecessor)
  uint8_t* smem = smem_all + (threadIdx.x >> 5) * route_warp_smem(E);
  // x (older than the router logits) is staged for the gate/up kernel before the wait;
  // the header is rewritten on every call so that nothing stale is taken for staged
  {
    const StageView sv = stage_view(ws, T, E, k, H);
    if (x != nullptr) {
      const __nv_bfloat16* xr = x + static_cast<int64_t>(t) * H;
      __half* dst = sv.x16 + static_cast<int64_t>(t) * H;
      float* xs = sv.xsum + static_cast<int64_t>(t) * (H / G);
      if (G == 128) stage_row<128>(xr, dst, xs, H, lane);
      else if (G == 64) stage_row<64>(xr, dst, xs, H, lane);
      else stage_row<32>(xr, dst, xs, H, lane);
    }
    if (t == 0 && lane == 0) {
      sv.tag[0] = reinterpret_cast<unsigned long long>(x);
      sv.tag[1] = x != nullptr ? stage_key(T, H, G) : 0ull;
    }
  }
  pdl_wait();   // the router logits come from the predecessor
  pdl_trigger();
  RouteView rv = route_view(ws, T, E, k);
  Q q{reinterpret_cast<float*>(smem), reinterpret_cast<int32_t*>(smem + E * 4)};
  int16_t* pos_l = reinterpret_cast<int16_t*>(smem + E * 8);
  int16_t* pos_r = pos_l + E + 2;
  const LT* row = logits + static_cast<int64_t>(t) * ldl;
  float sel_v = -INFINITY;   // lane r < k: value of the r-th selected expert
  int sel_i = 0;             //             and its index
  float mx = -INFINITY, z = 0.f;
  bool exact = E > 32 * ROUTE_MAXJ;
  float v[ROUTE_MAXJ];
  if (!exact) {
#pragma unroll
    for (int j = 0; j < ROUTE_MAXJ; ++j) {
      const int e = lane + 32 * j;
      v[j] = e < E ? to_f(row[e]) : -INFINITY;
    }
    const int rounds = k < E ? k + 1 : k;
    if constexpr (sizeof(LT) == 2) {
      // 16-bit logits: (value, index) packed in one word, the value's float_key with its
      // 12 low bits cleared (they are all zeros or all ones for a 16-bit type, so order
      // and equality of values are kept) above 4095 - index, so that each arg-max round
      // is one redux.sync; 0 is below every packed value and marks taken entries
      uint32_t pk[ROUTE_MAXJ];
      bool nan = false;
#pragma unroll
      for (int j = 0; j < ROUTE_MAXJ; ++j) {
        const int e = lane + 32 * j;
        nan |= e < E && isnan(v[j]);
        const float vc = v[j] == 0.f ? 0.f : v[j];   // -0 and +0 compare equal: one key
        pk[j] = e < E ? ((float_key(vc) & 0xFFFFF000u) | (0xFFFu - static_cast<uint32_t>(e))) : 0u;
      }
      if (__any_sync(0xffffffffu, nan)) {
        exact = true;   // NaN among the logits: the emulation reproduces their order
      } else {
        uint32_t prev = 0u;
        for (int r = 0; r < rounds; ++r) {
          uint32_t loc = 0u;
#pragma unroll
          for (int j = 0; j < ROUTE_MAXJ; ++j) loc = max(loc, pk[j]);
          const uint32_t best = __reduce_max_sync(0xffffffffu, loc);
          // a tie anywhere among the k+1 largest: use the exact emulation
          // (tie_order 0: only a tie at the k / k+1 boundary changes the selected set)
          if (r > 0 && (best >> 12) == (prev >> 12) && (tie_order || r == k)) { exact = true; break; }
          prev = best;
          const int e = 0xFFF - static_cast<int>(best & 0xFFFu);
          const uint32_t kv = best & 0xFFFFF000u;
          const float bv = __uint_as_float((kv & 0x80000000u) ? (kv ^ 0x80000000u) : ~(kv | 0xFFFu));
          if (r == 0) mx = bv;
          if (r < k && lane == r) { sel_v = bv; sel_i = e; }
          if ((e & 31) == lane) {
#pragma unroll
            for (int j = 0; j < ROUTE_MAXJ; ++j)
              if (j == (e >> 5)) pk[j] = 0u;
          }
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < ROUTE_MAXJ; ++j) mx = fmaxf(mx, v[j]);
      mx = warp_max(mx);
      unsigned taken = 0u;
      float prev = 0.f;
      for (int r = 0; r < rounds; ++r) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < ROUTE_MAXJ; ++j) {
          const int e = lane + 32 * j;
          if (e < E && !(taken >> j & 1u) && (bv < v[j] || bi == 0x7fffffff)) { bv = v[j]; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (oi != 0x7fffffff && (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
        }
        // a tie (or a NaN) anywhere among the k+1 largest: use the exact emulation
        if (r > 0 && !(prev > bv) && (tie_order || r == k || isnan(bv) || isnan(prev))) { exact = true; break; }
        prev = bv;
        if (r < k && lane == r) { sel_v = bv; sel_i = bi; }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
      }
    }
    if (!exact) {
#pragma unroll
      for (int j = 0; j < ROUTE_MAXJ; ++j)
        if (lane + 32 * j < E) z += __expf(v[j] - mx);
      z = warp_sum(z);
    }
  }
  if (exact) {
    // the row into shared memory: from the registers when the fast path loaded it
    const bool in_regs = E <= 32 * ROUTE_MAXJ;
    mx = -INFINITY;
    if (in_regs) {
#pragma unroll
      for (int j = 0; j < ROUTE_MAXJ; ++j) {
        const int e = lane + 32 * j;
        if (e < E) { q.v[e] = v[j]; q.i[e] = e; mx = fmaxf(mx, v[j]); }
      }
    } else {
      for (int e = lane; e < E; e += 32) {
        const float ve = to_f(row[e]);
        q.v[e] = ve;
        q.i[e] = e;
        mx = fmaxf(mx, ve);
      }
    }
    mx = warp_max(mx);
    z = 0.f;
    if (in_regs) {
#pragma unroll
      for (int j = 0; j < ROUTE_MAXJ; ++j)
        if (lane + 32 * j < E) z += __expf(v[j] - mx);
    } else {
      for (int e = lane; e < E; e += 32) z += __expf(q.v[e] - mx);
    }
    z = warp_sum(z);
    __syncwarp();
    warp_topk(q, E, k, pos_l, pos_r, lane);
    if (lane < k) { sel_v = q.v[lane]; sel_i = q.i[lane]; }
  }
  // renormalized weights of the selected (fused_ops.py:162-164)
  float p = 0.f;
  if (lane < k) p = __expf(sel_v - mx) / z;
  float ps = p;
  for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
  if (lane < k) {
    const float w = p / ps;
    rv.topk_idx[t * k + lane] = sel_i;
    rv.topk_w[t * k + lane] = act_is_f16 ? rnd<__half>(w) : rbf(w);
  }
  if (lane == 0) {
    float sg = 0.f;
    if (shared_col >= 0) {
      const float gl = to_f(row[shared_col]);
      sg = act_is_f16 ? rnd<__half>(sigmoid_f(gl)) : rbf(sigmoid_f(gl));
    }
    rv.shared_gate[t] = sg;
  }
}

// Expert -> (token, slot) lists of a block from its top-k indices idx[T * k]: the
// active experts in ascending id with their pair ranges (off), and in each range the
// pairs in ascending token.  Called by every thread of a CTA; scratch holds 3E ints,
// red 64 ints.  Outputs may live in shared or global memory.
__device__ void build_route_lists(const int* idx, int T, int E, int k, int lo, int* scratch, int* red,
                                  int* n_active, int* active, int* off, int* tok, int* slot) {
  const int nthr = blockDim.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // experts [lo, lo + E) of the routing, as local ids 0 .. E-1; pairs of other experts
  // (or invalid ids) are left out
  auto local = [&](int e) { return (e >= lo && e < lo + E) ? e - lo : -1; };
  int* cnt = scratch;                                  // [E] pairs per expert
  int* apos = scratch + E;                             // [E] next free position of each list
  unsigned* bits = reinterpret_cast<unsigned*>(scratch + 2 * E);   // [E] token bits of one 32-token chunk
  for (int e = threadIdx.x; e < E; e += nthr) cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < T * k; i += nthr) {
    const int e = local(idx[i]);
    if (e >= 0) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  // exclusive scans of (active flag, count) over experts: thread i owns a contiguous run
  const int per = (E + nthr - 1) / nthr;
  const int e0 = threadIdx.x * per, e1 = min(E, e0 + per);
  int my_a = 0, my_c = 0;
  for (int e = e0; e < e1; ++e) { my_a += cnt[e] > 0; my_c += cnt[e]; }
  int inc_a = my_a, inc_c = my_c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ua = __shfl_up_sync(0xffffffffu, inc_a, o), uc = __shfl_up_sync(0xffffffffu, inc_c, o);
    if (lane >= o) { inc_a += ua; inc_c += uc; }
  }
  if (lane == 31) { red[warp] = inc_a; red[32 + warp] = inc_c; }
  __syncthreads();
  int wa = 0, wc = 0;
  for (int w = 0; w < warp; ++w) { wa += red[w]; wc += red[32 + w]; }
  int na = wa + inc_a - my_a, o = wc + inc_c - my_c;
  for (int e = e0; e < e1; ++e) {
    if (cnt[e]) {
      active[na] = e;
      off[na] = o;
      apos[e] = o;
      o += cnt[e];
      ++na;
    }
  }
  if (threadIdx.x == nthr - 1) {
    off[na] = o;
    *n_active = na;
  }
  __syncthreads();
  // ranks within each expert's list, 32 tokens at a time
  for (int t0 = 0; t0 < T; t0 += 32) {
    const int tn = min(32, T - t0);
    for (int e = threadIdx.x; e < E; e += nthr) bits[e] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < tn * k; i += nthr) {
      const int e = local(idx[t0 * k + i]);
      if (e >= 0) atomicOr(&bits[e], 1u << (i / k));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < tn * k; i += nthr) {
      const int tl = i / k, s = i % k;
      const int e = local(idx[t0 * k + i]);
      if (e < 0) continue;
      const int at = apos[e] + __popc(bits[e] & ((1u << tl) - 1u));
      tok[at] = t0 + tl;
      slot[at] = s;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += nthr) apos[e] += __popc(bits[e]);
    __syncthreads();
  }
}

// Lists of the routing workspace (one CTA).  Dynamic smem: 3E + 64 ints.
// Lists of experts [lo, lo + ne) of a routing over E experts (local ids).
__global__ void __launch_bounds__(1024) route_lists_kernel(int T, int E, int k, int lo, int ne, void* ws) {
  extern __shared__ __align__(16) uint8_t smem[];
  pdl_wait();
  pdl_trigger();
  RouteView rv = route_view(ws, T, E, k);
  int* scratch = reinterpret_cast<int*>(smem);
  build_route_lists(rv.topk_idx, T, ne, k, lo, scratch, scratch + 3 * E, rv.n_active, rv.active, rv.pair_off,
                    rv.pair_tok, rv.pair_slot);
}

// ------------------------------------------------------------------ expert kernels
template <typename ET>
struct MoeArgs {
  const ET* x;              // [T, H] expert input (post-attention RMSNorm output)
  const uint8_t* gu;        // routed gate_up weights, expert e at gu + e * gu_stride
  const uint8_t* dn;        // routed down weights
  int64_t gu_stride, dn_stride;  // bytes per expert
  int64_t gu_ld, dn_ld;          // row stride in bytes (row format only)
  const uint8_t* sgu;       // shared expert gate|up ([2I, H]) and down ([H, I]), may be null
  const uint8_t* sdn;
  void* ws;                 // route workspace
  ET* hbuf;                 // [T*k + T, I]
  float* part;              // [T, k+1, H] raw expert outputs
  int T, H, I, E, k, has_shared;
  int e_lo, e_cnt;          // routed experts computed: [e_lo, e_lo + e_cnt) of the E, banks indexed e - e_lo
  int pairs_hint;           // expected routed pairs (0: T * k); picks the activation tile width
};

// Decode CTA slot -> (weights, number of pairs, pair list base); false if idle.
template <typename ET>
__device__ __forceinline__ bool slot_info(const MoeArgs<ET>& a, const RouteView& rv, int slot,
                                          bool up, const uint8_t*& w, int& npairs, int& pbase) {
  if (slot == 0) {
    if (!a.has_shared) return false;
    w = up ? a.sgu : a.sdn;
    npairs = a.T;
    pbase = -1;  // identity token list
    return true;
  }
  const int ai = slot - 1;
  if (ai >= *rv.n_active) return false;
  const int e = rv.active[ai];
  w = up ? a.gu + e * a.gu_stride : a.dn + e * a.dn_stride;
  pbase = rv.pair_off[ai];
  npairs = rv.pair_off[ai + 1] - pbase;
  return true;
}

// CTA = (expert slot, 4 intermediate tiles); warp w streams one whole row tile (gate
// rows of tile w/2 when w is even, the matching up rows when odd) over all of K through
// a PF-deep register ring, so every warp keeps PF chunks in flight for the CTA's whole
// life; gate/up pairs meet in shared memory for SiLU(gate) * up.
constexpr int UP_JT = 4;

template <class Fmt, int NT, int PF>
__global__ void __launch_bounds__(SG_WARPS * 32, 2) moe_up_kernel(MoeArgs<typename Fmt::ET> a) {
  using ET = typename Fmt::ET;
  constexpr int NTOK = NT * 8;
  __shared__ float gsm[UP_JT][NT * 4][32];
  pdl_wait();
  pdl_trigger();
  const RouteView rv = route_view(a.ws, a.T, a.E, a.k);
  const uint8_t* w;
  int npairs, pbase;
  if (!slot_info(a, rv, blockIdx.x, true, w, npairs, pbase)) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int jl = warp >> 1, role = warp & 1;
  const int jt = blockIdx.y * UP_JT + jl;  // intermediate tile
  const bool active = jt < a.I / 16;
  const int nch = a.H / Fmt::KCHUNK;
  const uint8_t* tile = w + Fmt::tile_offset(role * (a.I / 16) + (active ? jt : 0), a.H, a.gu_ld);
  const int gid = lane >> 2;
  for (int p0 = 0; p0 < npairs; p0 += NTOK) {
    const int np = min(NTOK, npairs - p0);
    XRows<ET, NT> xr;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int pi = p0 + min(j * 8 + gid, np - 1);
      const int tok = pbase < 0 ? pi : rv.pair_tok[pbase + pi];
      xr.r[j] = a.x + static_cast<int64_t>(tok) * a.H;
    }
    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    if (active) stream_tile<Fmt, NT, PF>(tile, a.gu_ld, 0, nch, lane, xr, acc);
    if (p0 > 0) __syncthreads();
    if (role == 0) {
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r) gsm[jl][j * 4 + r][lane] = acc[j][r];
    }
    __syncthreads();
    if (role == 1 && active) {
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int tl = frag_tok(lane, j, r);
          if (tl < np) {
            const float gr = rnd<ET>(gsm[jl][j * 4 + r][lane]), ur = rnd<ET>(acc[j][r]);
            const float h = rnd<ET>(rnd<ET>(silu_f(gr)) * ur);
            const int64_t hrow = pbase < 0 ? static_cast<int64_t>(a.T) * a.k + p0 + tl : pbase + p0 + tl;
            a.hbuf[hrow * a.I + jt * 16 + frag_row(lane, r)] = from_f<ET>(h);
          }
        }
    }
  }
}

template <class Fmt, int NT, int PF>
__global__ void __launch_bounds__(SG_WARPS * 32, 2) moe_down_kernel(MoeArgs<typename Fmt::ET> a) {
  using ET = typename Fmt::ET;
  constexpr int NTOK = NT * 8;
  pdl_wait();
  pdl_trigger();
  const RouteView rv = route_view(a.ws, a.T, a.E, a.k);
  const uint8_t* w;
  int npairs, pbase;
  if (!slot_info(a, rv, blockIdx.x, false, w, npairs, pbase)) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rt = blockIdx.y * SG_WARPS + warp;   // output row tile
  if (rt >= a.H / 16) return;
  const int nch = a.I / Fmt::KCHUNK;
  const uint8_t* tile = w + Fmt::tile_offset(rt, a.I, a.dn_ld);
  const int64_t hbase = pbase < 0 ? static_cast<int64_t>(a.T) * a.k : pbase;
  const int gid = lane >> 2;
  for (int p0 = 0; p0 < npairs; p0 += NTOK) {
    const int np = min(NTOK, npairs - p0);
    XRows<ET, NT> xr;
#pragma unroll
    for (int j = 0; j < NT; ++j) xr.r[j] = a.hbuf + (hbase + p0 + min(j * 8 + gid, np - 1)) * a.I;
    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    stream_tile<Fmt, NT, PF>(tile, a.dn_ld, 0, nch, lane, xr, acc);
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int tl = frag_tok(lane, j, r);
        if (tl < np) {
          int tok, slot;
          if (pbase < 0) { tok = p0 + tl; slot = a.k; }
          else { tok = rv.pair_tok[pbase + p0 + tl]; slot = rv.pair_slot[pbase + p0 + tl]; }
          a.part[(static_cast<int64_t>(tok) * (a.k + 1) + slot) * a.H + rt * 16 + frag_row(lane, r)] = acc[j][r];
        }
      }
  }
}

// ------------------------------------------------------------------ bulk-copy expert kernels
// Verify-block form (T <= 16 tokens) of the gate/up and down kernels: persistent CTAs
// (one per SM) of XT_UP_WARPS / XT_DN_WARPS warps, each warp streaming its weight tiles from HBM through
// its own ring of shared-memory stages with bulk copies (bulk_ring.cuh).  The expert
// inputs sit in shared memory, so the loop waits on nothing but the weight stream; the
// arithmetic (and its order) is that of moe_up_kernel / moe_down_kernel, so the results
// are the same bits.
constexpr int XT_UP_WARPS = 8;   // gate/up: whole (gate, up) tile pairs per warp
constexpr int XT_UP_CPS = 8;     // gate/up: W4 chunks per stage (at most)
constexpr int XT_DN_WARPS = 16;  // down: row blocks shared by the CTA
constexpr int XT_DN_CPS = 4;     // down: W4 chunks per stage (at most)
constexpr int XT_NST = 2;        // stages per warp ring
constexpr int XT_MAXT = 16;      // tokens of the block
constexpr int XT_BAR_BYTES = (16 * XT_NST * 8 + 127) / 128 * 128;   // up to 16 warps
constexpr int XT_PAD = 32;       // 16-bit elements of row padding: fragment loads hit distinct banks

// Route lists of the block, built in shared memory from the top-k indices.
struct XtRoute {
  int n_active;
  int idx[XT_MAXT * 16];
  int active[XT_MAXT * 16];
  int off[XT_MAXT * 16 + 1];
  int tok[XT_MAXT * 16];
  int slot[XT_MAXT * 16];
};

// Every thread of the CTA: the block's lists into r (scratch: 3E + 64 ints of shared
// memory).  With publish, the lists are also written to the routing workspace (for the
// host and for kernels that read the workspace lists).
__device__ __forceinline__ void xt_build_route(XtRoute& r, int* scratch, const RouteView& rv, int T, int E, int k,
                                               int lo, int ne, bool publish) {
  const int np = T * k;
  for (int i = threadIdx.x; i < np; i += blockDim.x) r.idx[i] = rv.topk_idx[i];
  __syncthreads();
  build_route_lists(r.idx, T, ne, k, lo, scratch, scratch + 3 * E, &r.n_active, r.active, r.off, r.tok, r.slot);
  if (publish) {
    const int na = r.n_active;
    if (threadIdx.x == 0) *rv.n_active = na;
    for (int i = threadIdx.x; i < na; i += blockDim.x) rv.active[i] = r.active[i];
    for (int i = threadIdx.x; i <= na; i += blockDim.x) rv.pair_off[i] = r.off[i];
    for (int i = threadIdx.x; i < np; i += blockDim.x) { rv.pair_tok[i] = r.tok[i]; rv.pair_slot[i] = r.slot[i]; }
  }
}

// Bytes of shared memory ahead of a bulk kernel's operand buffers: barriers, lists and
// the list-building scratch.
__host__ __device__ inline size_t xt_head_bytes(int E) {
  return XT_BAR_BYTES + (sizeof(XtRoute) + 127) / 128 * 128 + ((3 * static_cast<size_t>(E) + 64) * 4 + 127) / 128 * 128;
}

// Slot sl of the block: 0 the shared expert (when present), then the active experts.
template <typename A>
__device__ __forceinline__ void xt_slot(const A& a, const XtRoute& r, int sl, bool up, const uint8_t*& w,
                                        int& np, int& pbase) {
  if (a.has_shared && sl == 0) {
    w = up ? a.sgu : a.sdn;
    np = a.T;
    pbase = -1;
    return;
  }
  const int ai = sl - a.has_shared;
  const int e = r.active[ai];
  w = up ? a.gu + e * a.gu_stride : a.dn + e * a.dn_stride;
  pbase = r.off[ai];
  np = r.off[ai + 1] - pbase;
}

// Unit at position p of a round-robin deal of nu units over nw workers (worker w takes
// positions w, w + nw, ...).  Units 0 .. nh-1 are heavy (the shared expert's: all T
// tokens, two n-tiles of MMAs against one of a routed expert).  In natural order they
// land on the first workers, which also take a unit of the partial last round, and the
// launch waits for them; here they take the positions of the last full round whose
// workers get no unit of the partial round.  Only the assignment changes, not what a
// unit computes.
__device__ __forceinline__ int xt_unit_at(int p, int nu, int nw, int nh) {
  const int full = nu / nw, r0 = nu % nw;
  if (nh == 0 || full == 0 || r0 == 0 || r0 + nh > nw) return p;
  const int p0 = (full - 1) * nw + r0;
  if (p >= p0 && p < p0 + nh) return p - p0;
  return nh + (p < p0 ? p : p - nh);
}

struct XtArgs {
  MoeArgs<__nv_bfloat16> m;
  int32_t* status;      // g_moe_wait_status on the launching device
  long long limit;
  int dense_min;        // slots with at least this many pairs go to the tcgen05 kernels (0: none)
};

// Sticky status of the expert kernels' bounded waits (bulk_ring.cuh): set when a wait
// expired, read and cleared by qw_wait_status / qw_check_wait_status.
__device__ int32_t g_moe_wait_status;

static std::mutex g_moe_status_mu;
static int32_t* g_moe_status_ptr[64] = {};

int moe_wait_status_addr(int32_t** out) {
  return symbol_addr_cached(g_moe_wait_status, g_moe_status_ptr, 64, g_moe_status_mu, out,
                            "moe wait status address");
}

// Gate/up.  Unit = (slot, intermediate tile j): the gate row tile j then the up row tile
// I/16 + j, each cut into stages of up to XT_UP_CPS chunks; units are dealt round-robin
// to all warps (xt_unit_at: the shared expert's heavier units on warps with one unit
// fewer).  x [T, H] is staged once per CTA.  (Splitting a unit's K range over two warps
// was measured no faster, and would change the fp32 summation order against the
// streaming kernels that serve larger blocks.)
template <int G>
__global__ void __launch_bounds__(XT_UP_WARPS * 32, 1) moe_up_bulk_kernel(XtArgs args) {
  using Fmt = W4Fmt<G>;
  const MoeArgs<__nv_bfloat16>& a = args.m;
  extern __shared__ __align__(16) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  XtRoute& rt = *reinterpret_cast<XtRoute*>(smem + XT_BAR_BYTES);
  int* scratch = reinterpret_cast<int*>(smem + XT_BAR_BYTES + (sizeof(XtRoute) + 127) / 128 * 128);
  const int H = a.H, I = a.I, T = a.T;
  const int XS = H + XT_PAD;
  const int nch = H / G, cps = nch < XT_UP_CPS ? nch : XT_UP_CPS;
  __half* xs = reinterpret_cast<__half*>(smem + xt_head_bytes(a.E));
  float* xsum = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) + ((static_cast<size_t>(T) * XS * 2 + 127) / 128) * 128);
  uint8_t* ring_base = reinterpret_cast<uint8_t*>(xsum) + ((static_cast<size_t>(T) * nch * 4 + 127) / 128) * 128;
  const uint32_t sbytes = cps * Fmt::CHB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  WarpRing<XT_NST> ring{ring_base + warp * XT_NST * sbytes, bars + warp * XT_NST, sbytes, args.limit};
  if (lane == 0)
    for (int i = 0; i < XT_NST; ++i) mbar_init(ring.bar + i, 1);
  fence_barrier_init();
  const RouteView rv = route_view(a.ws, a.T, a.E, a.k);
  pdl_wait();   // the top-k indices and the staged x come from the predecessor (route)
  pdl_trigger();
  // the lists first: the weight copies below depend on them and are the long pole (the
  // activation copies issued ahead of them delayed the lists' loads)
  xt_build_route(rt, scratch, rv, T, a.E, a.k, a.e_lo, a.e_cnt, blockIdx.x == 0);
  __syncthreads();
  const int J = I / 16;
  const int nslots = a.has_shared + rt.n_active;
  const int nu = nslots * J;
  const int nh = a.has_shared && T > 8 ? J : 0;   // the shared expert's units: two n-tiles
  const int gw = blockIdx.x * XT_UP_WARPS + warp, nw = gridDim.x * XT_UP_WARPS;
  const int my_units = gw < nu ? (nu - 1 - gw) / nw + 1 : 0;
  // stage s of a unit: the gate chunks [s * hc, s * hc + hc) and the up chunks of the
  // same k range (two copies, the up half second); spu stages per unit
  const int hc = cps / 2, spu = nch / hc;
  const uint32_t hbytes = hc * Fmt::CHB;
  const int64_t tbytes = Fmt::tile_offset(1, H, 0);   // one row tile, all chunks
  const int Q = my_units * spu;
  // lane 0's copy cursor: the warp's unit cu_i, its stage cu_s, the unit's gate tile
  int cu_i = 0, cu_s = 0;
  const uint8_t* cu_w = nullptr;
  auto cursor_unit = [&]() {
    const int u = xt_unit_at(gw + cu_i * nw, nu, nw, nh);
    int np_, pb_;
    xt_slot(a, rt, u / J, true, cu_w, np_, pb_);
    cu_w += Fmt::tile_offset(u % J, H, 0);
  };
  auto issue_next = [&](int qq) {
    ring.issue2(qq, cu_w + cu_s * hbytes, cu_w + J * tbytes + cu_s * hbytes, hbytes);
    if (++cu_s == spu) {
      cu_s = 0;
      if (++cu_i < my_units) cursor_unit();
    }
  };
  if (lane == 0 && my_units > 0) {
    cursor_unit();
    for (int qq = 0; qq < XT_NST && qq < Q; ++qq) issue_next(qq);
  }
  // x -> shared memory (cp.async) while the first weight stages stream: as fp16 with its
  // group sums when the route kernel staged this x (qw_moe_route_x), else as bf16,
  // converted and summed below
  const StageView sv = stage_view(a.ws, T, a.E, a.k, H);
  const bool staged = sv.tag[0] == reinterpret_cast<unsigned long long>(a.x) && sv.tag[1] == stage_key(T, H, G);
  if (staged) {
    for (int i = threadIdx.x; i < T * (H / 8); i += blockDim.x) {
      const int r = i / (H / 8), c = (i % (H / 8)) * 8;
      cp_async16(xs + r * XS + c, sv.x16 + static_cast<int64_t>(r) * H + c, true);
    }
    if ((T * nch) % 4 == 0) {
      for (int i = threadIdx.x; i < T * nch / 4; i += blockDim.x) cp_async16(xsum + 4 * i, sv.xsum + 4 * i, true);
    } else {
      for (int i = threadIdx.x; i < T * nch; i += blockDim.x) xsum[i] = sv.xsum[i];
    }
  } else {
    for (int i = threadIdx.x; i < T * (H / 8); i += blockDim.x) {
      const int r = i / (H / 8), c = (i % (H / 8)) * 8;
      cp_async16(xs + r * XS + c, a.x + static_cast<int64_t>(r) * H + c, true);
    }
  }
  cp_async_commit();
  cp_async_wait<0>();
  // unstaged x: bf16 -> fp16 in place (each thread converts the vectors it copied), and
  // the per (token, K group) activation sums of the nibble MMA's offset term: with H a
  // multiple of 256 a warp holds whole groups of one row and sums them with shuffles
  if (staged) {
    __syncthreads();
  } else if (H % 256 == 0) {
    for (int i = threadIdx.x; i < T * (H / 8); i += blockDim.x) {
      const int r = i / (H / 8), sg = i % (H / 8);
      uint4* p = reinterpret_cast<uint4*>(xs + r * XS + sg * 8);
      const uint4 v = bf16x8_to_f16x8(*p);
      *p = v;
      const float xg = warp_group_xsum_f16<G>(sum8_f16(v), lane);
      if (sg % (G / 8) == 0) xsum[r * nch + sg / (G / 8)] = xg;
    }
    __syncthreads();
  } else {
    for (int i = threadIdx.x; i < T * (H / 8); i += blockDim.x) {
      uint4* p = reinterpret_cast<uint4*>(xs + (i / (H / 8)) * XS + (i % (H / 8)) * 8);
      *p = bf16x8_to_f16x8(*p);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < T * nch; i += blockDim.x) xsum[i] = group_xsum_f16<G>(xs + (i / nch) * XS + (i % nch) * G);
    __syncthreads();
  }
  const int gid = lane >> 2, tig = lane & 3;
  int q = 0;
  for (int i = 0; i < my_units; ++i) {
    const int u = xt_unit_at(gw + i * nw, nu, nw, nh), j = u % J;
    const uint8_t* w;
    int np, pb;
    xt_slot(a, rt, u / J, true, w, np, pb);
    const bool two = np > 8;
    const __half* xr[2];
    const float* xq[2][2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int idx = min(nt * 8 + gid, np - 1);
      xr[nt] = xs + (pb < 0 ? idx : rt.tok[pb + idx]) * XS;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int ci = min(nt * 8 + 2 * tig + e, np - 1);
        xq[nt][e] = xsum + (pb < 0 ? ci : rt.tok[pb + ci]) * nch;
      }
    }
    float accg[2][4], accu[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) accg[nt][r] = accu[nt][r] = 0.f;
    for (int s = 0; s < spu; ++s, ++q) {
      if (!ring.wait(q, args.status)) {
        if (lane == 0) ring.drain(q + 1, min(q + XT_NST, Q));
        return;
      }
      const uint8_t* st = ring.stage(q);
      // one n-tile of the stage, four chunk pairs at a time (eight independent MMA chains)
      auto tile = [&](const __half* xrn, const float* q0, const float* q1, float(&ag)[4], float(&au)[4]) {
        int c = 0;
        for (; c + 4 <= hc; c += 4)
          w4n_smem_pairs<G, 4>(st + c * Fmt::CHB, st + hbytes + c * Fmt::CHB, xrn, (s * hc + c) * G, q0, q1,
                               s * hc + c, lane, ag, au);
        for (; c < hc; ++c)
          w4n_smem_pair<G>(st + c * Fmt::CHB, st + hbytes + c * Fmt::CHB, xrn, (s * hc + c) * G, q0, q1, s * hc + c,
                           lane, ag, au);
      };
      tile(xr[0], xq[0][0], xq[0][1], accg[0], accu[0]);
      if (two) tile(xr[1], xq[1][0], xq[1][1], accg[1], accu[1]);
      __syncwarp();
      if (lane == 0 && q + XT_NST < Q) issue_next(q + XT_NST);
    }
    // h = silu(gate) * up in the reference's rounding order
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int tl = frag_tok(lane, nt, r);
        if (tl < np) {
          const float gr = rbf(accg[nt][r]), ur = rbf(accu[nt][r]);
          const float h = rbf(rbf(silu_f(gr)) * ur);
          const int64_t hrow = pb < 0 ? static_cast<int64_t>(T) * a.k + tl : pb + tl;
          // h is a bf16 value; stored as fp16 (exact) for the bulk down kernel's operand
          reinterpret_cast<__half*>(a.hbuf)[hrow * I + j * 16 + frag_row(lane, r)] = __float2half_rn(h);
        }
      }
  }
}

// Down.  Unit = (slot, block of XT_DN_WARPS * spw row tiles); the CTA's warps share the
// unit, each streaming spw... stages of tiles; the unit's rows of h are staged in shared
// memory (three buffers across units).  Units go to CTAs round-robin (xt_unit_at: the
// shared expert's heavier units on CTAs with one unit fewer).
template <int G>
__global__ void __launch_bounds__(XT_DN_WARPS * 32, 1) moe_down_bulk_kernel(XtArgs args, int tiles_per_stage,
                                                                         int stages_per_warp) {
  using Fmt = W4Fmt<G>;
  const MoeArgs<__nv_bfloat16>& a = args.m;
  extern __shared__ __align__(16) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  XtRoute& rt = *reinterpret_cast<XtRoute*>(smem + XT_BAR_BYTES);
  int* scratch = reinterpret_cast<int*>(smem + XT_BAR_BYTES + (sizeof(XtRoute) + 127) / 128 * 128);
  const int H = a.H, I = a.I, T = a.T;
  const int HS = I + XT_PAD;
  __half* hs = reinterpret_cast<__half*>(smem + xt_head_bytes(a.E));
  const size_t hbytes = ((static_cast<size_t>(XT_MAXT) * HS * 2 + 127) / 128) * 128;
  uint8_t* ring_base = reinterpret_cast<uint8_t*>(hs) + 3 * hbytes;
  const int cpt = I / G;                         // chunks per row tile
  const int tps = tiles_per_stage, spw = stages_per_warp;
  const uint32_t sbytes = tps * cpt * Fmt::CHB;
  const int rb_tiles = XT_DN_WARPS * spw * tps;     // row tiles per unit
  const int nrb = (H / 16) / rb_tiles;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  WarpRing<XT_NST> ring{ring_base + warp * XT_NST * sbytes, bars + warp * XT_NST, sbytes, args.limit};
  if (lane == 0)
    for (int i = 0; i < XT_NST; ++i) mbar_init(ring.bar + i, 1);
  fence_barrier_init();
  const RouteView rv = route_view(a.ws, a.T, a.E, a.k);
  xt_build_route(rt, scratch, rv, T, a.E, a.k, a.e_lo, a.e_cnt, false);
  __syncthreads();
  const int nslots = a.has_shared + rt.n_active;
  const int nu = nslots * nrb;
  const int nh = a.has_shared && T > 8 ? nrb : 0;   // the shared expert's units: two n-tiles
  const int my_units = blockIdx.x < nu ? (nu - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int Q = my_units * spw;
  auto src = [&](int q) -> const uint8_t* {
    const int u = xt_unit_at(blockIdx.x + (q / spw) * gridDim.x, nu, gridDim.x, nh), l = q % spw;
    const uint8_t* w;
    int np, pb;
    xt_slot(a, rt, u / nrb, false, w, np, pb);
    const int tile = (u % nrb) * rb_tiles + (warp * spw + l) * tps;
    return w + Fmt::tile_offset(tile, I, 0);
  };
  if (lane == 0)
    for (int q = 0; q < XT_NST && q < Q; ++q) ring.issue(q, src(q), sbytes);
  // h rows of unit i -> buffer i % 3: it is restaged (for unit i + 3) only after every
  // warp has passed the barrier of unit i + 1, so units need one barrier each
  auto stage_h = [&](int i) {
    const int u = xt_unit_at(blockIdx.x + i * gridDim.x, nu, gridDim.x, nh);
    const uint8_t* w;
    int np, pb;
    xt_slot(a, rt, u / nrb, false, w, np, pb);
    const int64_t hb = pb < 0 ? static_cast<int64_t>(T) * a.k : pb;
    __half* dst = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(hs) + (i % 3) * hbytes);
    const __half* hsrc = reinterpret_cast<const __half*>(a.hbuf);
    for (int e = threadIdx.x; e < np * (I / 8); e += blockDim.x) {
      const int r = e / (I / 8), c = (e % (I / 8)) * 8;
      cp_async16(dst + r * HS + c, hsrc + (hb + r) * I + c, true);
    }
  };
  pdl_wait();   // h comes from the predecessor (gate/up); the lists and weights do not
  pdl_trigger();
  // With at most three units (the usual case) every unit's h rows fit the three buffers:
  // they are staged once, behind one barrier, and the warps then run their units
  // without CTA barriers (a barrier per unit made each unit wait for the CTA's slowest
  // weight copy).  Otherwise unit i + 1 is staged while unit i runs.
  const bool h_once = my_units <= 3;
  if (h_once) {
    for (int i = 0; i < my_units; ++i) stage_h(i);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
  } else {
    stage_h(0);
    cp_async_commit();
  }
  const int gid = lane >> 2;
  int q = 0;
  bool ok = true;
  for (int i = 0; i < my_units; ++i) {
    if (!h_once) {
      if (i + 1 < my_units) stage_h(i + 1);
      cp_async_commit();
      cp_async_wait<1>();
      __syncthreads();
    }
    const int u = xt_unit_at(blockIdx.x + i * gridDim.x, nu, gridDim.x, nh);
    const uint8_t* w;
    int np, pb;
    xt_slot(a, rt, u / nrb, false, w, np, pb);
    const bool two = np > 8;
    const __half* hbuf_s = reinterpret_cast<const __half*>(reinterpret_cast<const uint8_t*>(hs) + (i % 3) * hbytes);
    const __half* xr[2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) xr[nt] = hbuf_s + min(nt * 8 + gid, np - 1) * HS;
    for (int l = 0; l < spw && ok; ++l, ++q) {
      if (!ring.wait(q, args.status)) {
        if (lane == 0) ring.drain(q + 1, min(q + XT_NST, Q));
        ok = false;
        break;
      }
      const uint8_t* st = ring.stage(q);
      for (int t = 0; t < tps; ++t) {
        float acc[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
        w4_smem_run<G>(st + t * cpt * Fmt::CHB, cpt, xr, 0, lane, two, acc);
        const int row0 = ((u % nrb) * rb_tiles + (warp * spw + l) * tps + t) * 16;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int tl = frag_tok(lane, nt, r);
            if (tl < np) {
              int tok, slot;
              if (pb < 0) { tok = tl; slot = a.k; }
              else { tok = rt.tok[pb + tl]; slot = rt.slot[pb + tl]; }
              a.part[(static_cast<int64_t>(tok) * (a.k + 1) + slot) * H + row0 + frag_row(lane, r)] = acc[nt][r];
            }
          }
      }
      __syncwarp();
      if (lane == 0 && q + XT_NST < Q) ring.issue(q + XT_NST, src(q + XT_NST), sbytes);
    }
    // a warp that timed out keeps staging and taking part in the units' barriers
  }
  cp_async_wait<0>();
}

// ------------------------------------------------------------------ expert-parallel window
// (the exchange itself is described with its kernels at the end of this file)
constexpr int EP_MAX_RANKS = 64;
constexpr long long EP_PEER_WAIT_LIMIT = 1ll << 34;   // cycles (~9 s): a peer's host may lag in eager use

// Arrival counters: every exchange adds exactly EP_ROUND to the receiving counter of
// each (sender, receiver) pair -- one per row as it lands, with release semantics, and
// EP_ROUND - rows in one add from the sender, which knows the count -- so after exchange
// n the counter is n * EP_ROUND, and no partial sum of exchange n reaches it.
constexpr unsigned long long EP_ROUND = 1ull << 20;

struct EpWin {
  int32_t* hdr;                 // [0] epoch of the last closed exchange, [3] ticket, [4] broken
  unsigned long long* dcnt;     // [64] rows (and count messages) arrived from source s
  unsigned long long* ccnt;     // [64] results arrived from expert owner d
  int32_t* count;               // [64] rows source s sent in the current exchange
  int32_t* meta;
  __nv_bfloat16* rows;
  __nv_bfloat16* back;
};

constexpr int EP_HEAD_BYTES = 2048;

__host__ __device__ inline int64_t ep_window_bytes(int G, int cap, int H) {
  int64_t off = EP_HEAD_BYTES;
  off += align256(static_cast<int64_t>(G) * cap * 4);
  off += align256(static_cast<int64_t>(G) * cap * H * 2);
  off += align256(static_cast<int64_t>(cap) * H * 2);
  return off;
}

__host__ __device__ inline EpWin ep_win(const void* base, int G, int cap, int H) {
  uint8_t* p = static_cast<uint8_t*>(const_cast<void*>(base));
  EpWin w;
  w.hdr = reinterpret_cast<int32_t*>(p);
  w.dcnt = reinterpret_cast<unsigned long long*>(p + 256);
  w.ccnt = w.dcnt + EP_MAX_RANKS;
  w.count = reinterpret_cast<int32_t*>(p + 256 + 2 * EP_MAX_RANKS * 8);
  int64_t off = EP_HEAD_BYTES;
  w.meta = reinterpret_cast<int32_t*>(p + off);
  off += align256(static_cast<int64_t>(G) * cap * 4);
  w.rows = reinterpret_cast<__nv_bfloat16*>(p + off);
  off += align256(static_cast<int64_t>(G) * cap * H * 2);
  w.back = reinterpret_cast<__nv_bfloat16*>(p + off);
  return w;
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Add to a (peer's) counter, ordered after every store this thread has observed.
__device__ __forceinline__ void red_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}

// Bounded wait (one thread) until *counter reaches `want` (added by peer GPUs).  On
// expiry -- or when an earlier wait of this window expired (hdr[4]) -- records the
// timeout in the sticky status and returns false, so a lost peer costs one limit, not
// one per wait.
__device__ bool ep_wait_count(const unsigned long long* counter, unsigned long long want, int32_t* hdr) {
  if (ld_acquire_sys(counter) >= want) return true;
  const long long t0 = clock64();
  while (ld_acquire_sys(counter) < want) {
    if (*reinterpret_cast<volatile int32_t*>(hdr + 4) != 0 || clock64() - t0 > EP_PEER_WAIT_LIMIT) {
      atomicOr(&g_moe_wait_status, QW_DEVICE_TIMEOUT);
      *reinterpret_cast<volatile int32_t*>(hdr + 4) = 1;
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// The CTA that finishes last (ticket wraps to 0 for the next launch); used to close an
// exchange after every CTA of the kernel has read what it needs.
__device__ __forceinline__ bool ep_last_cta(int32_t* ticket) {
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicInc(reinterpret_cast<unsigned*>(ticket), gridDim.x - 1) == gridDim.x - 1;
  }
  __syncthreads();
  return s_last != 0;
}

// ------------------------------------------------------------------ grouped bulk kernels
// The bulk-copy gate/up and down kernels for any number of tokens (T > 16, and the rows an
// expert-parallel rank receives): the expert lists come from the routing workspace
// (qw_moe_route_lists or the receive routing), and an expert's tokens are taken in
// chunks of at most 16.  Work is cut into items of whole weight-tile groups of one
// (expert slot, token chunk) "segment"; a CTA takes a contiguous range of items and
// stages a segment's activation rows in shared memory once, when the segment changes.
// Per row tile and token the MMA sequence and the epilogue are those of the bulk
// kernels, so every output has their bits.
constexpr int GR_CHUNK = 16;          // tokens per segment, at most
// dynamic shared memory of the grouped kernels, at most: the CTA limit less room for the
// few bytes of static shared memory the expert-parallel epilogue uses
constexpr size_t GR_SMEM_LIMIT = 227 * 1024 - 256;
constexpr int GR_MAX_SLOTS = 1 + 512;  // shared expert + active experts

// Segment table in shared memory: for every slot its pair count and the first item of
// each slot, so an item index maps to (slot, chunk, tile block) by a binary search.
struct GrTable {
  int nslots, total;          // slots, items (or units) in all
  int first[GR_MAX_SLOTS + 1];  // first item of slot s; first[nslots] = total
};

template <typename ET>
__device__ __forceinline__ int gr_pairs(const MoeArgs<ET>& a, const RouteView& rv, int slot) {
  if (a.has_shared && slot == 0) return a.T;
  const int ai = slot - a.has_shared;
  return rv.pair_off[ai + 1] - rv.pair_off[ai];
}

// The tcgen05 kernels take an expert's pairs in tiles of this many, and run at all only
// when the routed experts with at least dense_min pairs make this many gate/up items
// (tiles x 64-column blocks): fewer would run serially on a few SMs after the grouped
// kernels and cost more than they save (measured).
constexpr int TC_N = 128;
constexpr int TC_MIN_ITEMS = 128;

// Every thread (a CTA-wide vote): do the dense experts of this routing fill the GPU?
// The grouped and the tcgen05 kernels decide alike from the same counts.
template <typename ET>
__device__ bool dense_path_fills(const MoeArgs<ET>& a, const RouteView& rv, int dense_min) {
  __shared__ int tiles;
  if (threadIdx.x == 0) tiles = 0;
  __syncthreads();
  const int ns = a.has_shared + *rv.n_active;
  int mine = 0;
  for (int sl = a.has_shared + threadIdx.x; sl < ns; sl += blockDim.x) {
    const int np = gr_pairs(a, rv, sl);
    if (np >= dense_min) mine += (np + TC_N - 1) / TC_N;
  }
  if (mine) atomicAdd(&tiles, mine);
  __syncthreads();
  return tiles * (a.I / 64) >= TC_MIN_ITEMS;
}

// Every thread: the table with `per` items per (slot, chunk of `chunk` pairs).  A routed
// expert's slot with at least dense_min pairs (dense_min > 0, and the dense experts
// filling the GPU) belongs to the tcgen05 kernels: with
// dense false it gets no items here, with dense true only such slots get items.  The
// slots' item counts load in parallel; warp 0 scans them 32 at a time.
template <typename ET>
__device__ void gr_build_table(GrTable& tb, const MoeArgs<ET>& a, const RouteView& rv, int per, int dense_min = 0,
                               bool dense = false, int chunk = GR_CHUNK) {
  const int ns = a.has_shared + *rv.n_active;
  if (dense_min > 0 && !dense_path_fills(a, rv, dense_min)) dense_min = 0;
  for (int sl = threadIdx.x; sl < ns; sl += blockDim.x) {
    const int np = gr_pairs(a, rv, sl);
    const bool is_dense = dense_min > 0 && !(a.has_shared && sl == 0) && np >= dense_min;
    tb.first[sl] = is_dense == dense ? (np + chunk - 1) / chunk * per : 0;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int carry = 0;
    for (int base = 0; base < ns; base += 32) {
      const int v = base + lane < ns ? tb.first[base + lane] : 0;
      int inc = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += u;
      }
      if (base + lane < ns) tb.first[base + lane] = carry + inc - v;
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) {
      tb.first[ns] = carry;
      tb.nslots = ns;
      tb.total = carry;
    }
  }
  __syncthreads();
}

__device__ __forceinline__ int gr_slot_of(const GrTable& tb, int item) {
  int lo = 0, hi = tb.nslots - 1;   // the last slot whose first item <= item
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tb.first[mid] <= item) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Segment of item `item`: slot, chunk, item within the (slot, chunk), the weights, the
// segment's token count and the base of its pair list (-1: identity, shared expert).
template <typename ET>
__device__ __forceinline__ void gr_item(const GrTable& tb, const MoeArgs<ET>& a, const RouteView& rv, int item,
                                        int per, bool up, int& slot, int& chunk, int& sub, const uint8_t*& w,
                                        int& np, int& pbase) {
  slot = gr_slot_of(tb, item);
  const int r = item - tb.first[slot];
  chunk = r / per;
  sub = r % per;
  const int npairs = gr_pairs(a, rv, slot);
  np = min(GR_CHUNK, npairs - chunk * GR_CHUNK);
  if (a.has_shared && slot == 0) {
    w = up ? a.sgu : a.sdn;
    pbase = -1;
  } else {
    const int ai = slot - a.has_shared;
    const int e = rv.active[ai];
    w = up ? a.gu + e * a.gu_stride : a.dn + e * a.dn_stride;
    pbase = rv.pair_off[ai];
  }
}

// Gate/up.  Item = (slot, chunk, block of XT_UP_WARPS intermediate tiles): warp w takes
// tile block * XT_UP_WARPS + w (I / 16 a multiple of the warp count).
template <int G>
__global__ void __launch_bounds__(XT_UP_WARPS * 32, 1) moe_up_grouped_kernel(XtArgs args) {
  using Fmt = W4Fmt<G>;
  const MoeArgs<__nv_bfloat16>& a = args.m;
  extern __shared__ __align__(16) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  GrTable& tb = *reinterpret_cast<GrTable*>(smem + XT_BAR_BYTES);
  const int H = a.H, I = a.I;
  const int XS = H + XT_PAD;
  const int nch = H / G, cps = nch < XT_UP_CPS ? nch : XT_UP_CPS;
  __half* xs = reinterpret_cast<__half*>(smem + XT_BAR_BYTES + (sizeof(GrTable) + 127) / 128 * 128);
  float* xsum = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) +
                                         ((static_cast<size_t>(GR_CHUNK) * XS * 2 + 127) / 128) * 128);
  uint8_t* ring_base = reinterpret_cast<uint8_t*>(xsum) + ((static_cast<size_t>(GR_CHUNK) * nch * 4 + 127) / 128) * 128;
  const uint32_t sbytes = cps * Fmt::CHB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  WarpRing<XT_NST> ring{ring_base + warp * XT_NST * sbytes, bars + warp * XT_NST, sbytes, args.limit};
  if (lane == 0)
    for (int i = 0; i < XT_NST; ++i) mbar_init(ring.bar + i, 1);
  fence_barrier_init();
  const RouteView rv = route_view(a.ws, a.T, a.E, a.k);
  pdl_wait();   // the lists (and the received rows) come from the predecessor
  pdl_trigger();
  const int J = I / 16, per = J / XT_UP_WARPS;
  gr_build_table(tb, a, rv, per, args.dense_min);
  const int n_items = tb.total;
  const int i0 = static_cast<int>(static_cast<int64_t>(n_items) * blockIdx.x / gridDim.x);
  const int i1 = static_cast<int>(static_cast<int64_t>(n_items) * (blockIdx.x + 1) / gridDim.x);
  const int hc = cps / 2, spu = nch / hc;
  const uint32_t hbytes = hc * Fmt::CHB;
  const int64_t tbytes = Fmt::tile_offset(1, H, 0);
  const int Q = (i1 - i0) * spu;
  // lane 0's copy cursor over this warp's units (one per item)
  int cu_i = i0, cu_s = 0;
  const uint8_t* cu_w = nullptr;
  auto cursor_unit = [&]() {
    int sl, ch, sub, np_, pb_;
    gr_item(tb, a, rv, cu_i, per, true, sl, ch, sub, cu_w, np_, pb_);
    cu_w += Fmt::tile_offset(sub * XT_UP_WARPS + warp, H, 0);
  };
  auto issue_next = [&](int qq) {
    ring.issue2(qq, cu_w + cu_s * hbytes, cu_w + J * tbytes + cu_s * hbytes, hbytes);
    if (++cu_s == spu) {
      cu_s = 0;
      if (++cu_i < i1) cursor_unit();
    }
  };
  if (lane == 0 && i1 > i0) {
    cursor_unit();
    for (int qq = 0; qq < XT_NST && qq < Q; ++qq) issue_next(qq);
  }
  const int gid = lane >> 2, tig = lane & 3;
  int q = 0, seg_slot = -1, seg_chunk = -1;
  bool ok = true;
  for (int it = i0; it < i1; ++it) {
    int sl, ch, sub, np, pb;
    const uint8_t* w;
    gr_item(tb, a, rv, it, per, true, sl, ch, sub, w, np, pb);
    if (sl != seg_slot || ch != seg_chunk) {
      // a new segment: its rows as fp16 and their group sums (after every warp is done
      // with the previous segment's)
      __syncthreads();
      for (int i = threadIdx.x; i < np * (H / 8); i += blockDim.x) {
        const int r = i / (H / 8), c = (i % (H / 8)) * 8;
        const int pi = ch * GR_CHUNK + r;
        const int tok = pb < 0 ? pi : rv.pair_tok[pb + pi];
        cp_async16(xs + r * XS + c, a.x + static_cast<int64_t>(tok) * H + c, true);
      }
      cp_async_commit();
      cp_async_wait<0>();
      if (H % 256 == 0) {
        for (int i = threadIdx.x; i < np * (H / 8); i += blockDim.x) {
          const int r = i / (H / 8), sg = i % (H / 8);
          uint4* p = reinterpret_cast<uint4*>(xs + r * XS + sg * 8);
          const uint4 v = bf16x8_to_f16x8(*p);
          *p = v;
          const float xg = warp_group_xsum_f16<G>(sum8_f16(v), lane);
          if (sg % (G / 8) == 0) xsum[r * nch + sg / (G / 8)] = xg;
        }
        __syncthreads();
      } else {
        for (int i = threadIdx.x; i < np * (H / 8); i += blockDim.x) {
          uint4* p = reinterpret_cast<uint4*>(xs + (i / (H / 8)) * XS + (i % (H / 8)) * 8);
          *p = bf16x8_to_f16x8(*p);
        }
        __syncthreads();
        for (int i = threadIdx.x; i < np * nch; i += blockDim.x)
          xsum[i] = group_xsum_f16<G>(xs + (i / nch) * XS + (i % nch) * G);
        __syncthreads();
      }
      seg_slot = sl;
      seg_chunk = ch;
    }
    if (!ok) continue;   // a warp that timed out still takes part in the segment barriers
    const int j = sub * XT_UP_WARPS + warp;
    const bool two = np > 8;
    const __half* xr[2];
    const float* xq[2][2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      xr[nt] = xs + min(nt * 8 + gid, np - 1) * XS;
#pragma unroll
      for (int e = 0; e < 2; ++e) xq[nt][e] = xsum + min(nt * 8 + 2 * tig + e, np - 1) * nch;
    }
    float accg[2][4], accu[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) accg[nt][r] = accu[nt][r] = 0.f;
    for (int s = 0; s < spu; ++s, ++q) {
      if (!ring.wait(q, args.status)) {
        if (lane == 0) ring.drain(q + 1, min(q + XT_NST, Q));
        ok = false;
        break;
      }
      const uint8_t* st = ring.stage(q);
      // one n-tile of the stage, four chunk pairs at a time (eight independent MMA chains)
      auto tile = [&](const __half* xrn, const float* q0, const float* q1, float(&ag)[4], float(&au)[4]) {
        int c = 0;
        for (; c + 4 <= hc; c += 4)
          w4n_smem_pairs<G, 4>(st + c * Fmt::CHB, st + hbytes + c * Fmt::CHB, xrn, (s * hc + c) * G, q0, q1,
                               s * hc + c, lane, ag, au);
        for (; c < hc; ++c)
          w4n_smem_pair<G>(st + c * Fmt::CHB, st + hbytes + c * Fmt::CHB, xrn, (s * hc + c) * G, q0, q1, s * hc + c,
                           lane, ag, au);
      };
      tile(xr[0], xq[0][0], xq[0][1], accg[0], accu[0]);
      if (two) tile(xr[1], xq[1][0], xq[1][1], accg[1], accu[1]);
      __syncwarp();
      if (lane == 0 && q + XT_NST < Q) issue_next(q + XT_NST);
    }
    if (!ok) continue;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int tl = frag_tok(lane, nt, r);
        if (tl < np) {
          const float gr = rbf(accg[nt][r]), ur = rbf(accu[nt][r]);
          const float h = rbf(rbf(silu_f(gr)) * ur);
          const int pi = ch * GR_CHUNK + tl;
          const int64_t hrow = pb < 0 ? static_cast<int64_t>(a.T) * a.k + pi : pb + pi;
          reinterpret_cast<__half*>(a.hbuf)[hrow * I + j * 16 + frag_row(lane, r)] = __float2half_rn(h);
        }
      }
  }
}

// Where an expert-parallel rank's down projection sends its results: row r of the
// receiving routing came from rank r / cap (window meta[r] = (pair << 9) | expert); its
// output goes, as bf16, to row `pair` of that rank's `back`.
struct EpSend {
  void* window;                      // this rank's window (null: plain f32 outputs)
  const unsigned long long* peers;   // every rank's window
  int G, rank, cap;
};

// Down.  Unit = (slot, chunk, block of XT_DN_WARPS * spw row tiles), as in the bulk down
// kernel; units go to CTAs round-robin and the unit's h rows are staged per unit.  With
// an EpSend window the unit's outputs are rounded to bf16 (the precision the combine
// reads), gathered in shared memory and stored with 16-byte stores straight into the
// source ranks' windows; the last CTA then raises this rank's combine flag in every
// window.
template <int G, bool EP>
__global__ void __launch_bounds__(XT_DN_WARPS * 32, 1) moe_down_grouped_kernel(XtArgs args, int tiles_per_stage,
                                                                            int stages_per_warp, EpSend ep) {
  using Fmt = W4Fmt<G>;
  const MoeArgs<__nv_bfloat16>& a = args.m;
  extern __shared__ __align__(16) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  GrTable& tb = *reinterpret_cast<GrTable*>(smem + XT_BAR_BYTES);
  const int H = a.H, I = a.I, T = a.T;
  const int HS = I + XT_PAD;
  __half* hs = reinterpret_cast<__half*>(smem + XT_BAR_BYTES + (sizeof(GrTable) + 127) / 128 * 128);
  const size_t hbytes = ((static_cast<size_t>(GR_CHUNK) * HS * 2 + 127) / 128) * 128;
  const int cpt = I / G;
  const int tps = tiles_per_stage, spw = stages_per_warp;
  const uint32_t sbytes = tps * cpt * Fmt::CHB;
  const int rb_tiles = XT_DN_WARPS * spw * tps;
  // EP: the unit's bf16 outputs [GR_CHUNK][rb_tiles * 16 (+8)] before they leave
  const int OS = rb_tiles * 16 + 8;
  __nv_bfloat16* osm = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(hs) + 3 * hbytes);
  const size_t obytes = EP ? ((static_cast<size_t>(GR_CHUNK) * OS * 2 + 127) / 128) * 128 : 0;
  uint8_t* ring_base = reinterpret_cast<uint8_t*>(hs) + 3 * hbytes + obytes;
  const int nrb = (H / 16) / rb_tiles;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  WarpRing<XT_NST> ring{ring_base + warp * XT_NST * sbytes, bars + warp * XT_NST, sbytes, args.limit};
  if (lane == 0)
    for (int i = 0; i < XT_NST; ++i) mbar_init(ring.bar + i, 1);
  fence_barrier_init();
  const RouteView rv = route_view(a.ws, a.T, a.E, a.k);
  pdl_wait();   // h comes from the predecessor (gate/up); the lists from earlier kernels
  pdl_trigger();
  if constexpr (EP) {
    // every received row returns to its source as nrb pieces (one per unit), each
    // counted on arrival; the complement to EP_ROUND goes now, from CTA 0
    if (blockIdx.x == 0 && threadIdx.x < ep.G) {
      const EpWin me = ep_win(ep.window, ep.G, ep.cap, H);
      const unsigned long long pieces = static_cast<unsigned long long>(__ldcg(me.count + threadIdx.x)) * nrb;
      red_release_sys(ep_win(reinterpret_cast<const void*>(ep.peers[threadIdx.x]), ep.G, ep.cap, H).ccnt + ep.rank,
                      EP_ROUND - pieces);
    }
  }
  gr_build_table(tb, a, rv, nrb, args.dense_min);
  const int nu = tb.total;
  const int my_units = blockIdx.x < nu ? (nu - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int Q = my_units * spw;
  auto src = [&](int q) -> const uint8_t* {
    const int u = blockIdx.x + (q / spw) * gridDim.x, l = q % spw;
    int sl, ch, sub, np, pb;
    const uint8_t* w;
    gr_item(tb, a, rv, u, nrb, false, sl, ch, sub, w, np, pb);
    const int tile = sub * rb_tiles + (warp * spw + l) * tps;
    return w + Fmt::tile_offset(tile, I, 0);
  };
  if (lane == 0)
    for (int q = 0; q < XT_NST && q < Q; ++q) ring.issue(q, src(q), sbytes);
  auto stage_h = [&](int i) {
    const int u = blockIdx.x + i * gridDim.x;
    int sl, ch, sub, np, pb;
    const uint8_t* w;
    gr_item(tb, a, rv, u, nrb, false, sl, ch, sub, w, np, pb);
    const int64_t hb = (pb < 0 ? static_cast<int64_t>(T) * a.k : pb) + ch * GR_CHUNK;
    __half* dst = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(hs) + (i % 3) * hbytes);
    const __half* hsrc = reinterpret_cast<const __half*>(a.hbuf);
    for (int e = threadIdx.x; e < np * (I / 8); e += blockDim.x) {
      const int r = e / (I / 8), c = (e % (I / 8)) * 8;
      cp_async16(dst + r * HS + c, hsrc + (hb + r) * I + c, true);
    }
  };
  if (my_units > 0) stage_h(0);
  cp_async_commit();
  const int gid = lane >> 2;
  int q = 0;
  bool ok = true;
  for (int i = 0; i < my_units; ++i) {
    if (i + 1 < my_units) stage_h(i + 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int u = blockIdx.x + i * gridDim.x;
    int sl, ch, sub, np, pb;
    const uint8_t* w;
    gr_item(tb, a, rv, u, nrb, false, sl, ch, sub, w, np, pb);
    const bool two = np > 8;
    const __half* hbuf_s = reinterpret_cast<const __half*>(reinterpret_cast<const uint8_t*>(hs) + (i % 3) * hbytes);
    const __half* xr[2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) xr[nt] = hbuf_s + min(nt * 8 + gid, np - 1) * HS;
    for (int l = 0; l < spw && ok; ++l, ++q) {
      if (!ring.wait(q, args.status)) {
        if (lane == 0) ring.drain(q + 1, min(q + XT_NST, Q));
        ok = false;
        break;
      }
      const uint8_t* st = ring.stage(q);
      for (int t = 0; t < tps; ++t) {
        float acc[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
        w4_smem_run<G>(st + t * cpt * Fmt::CHB, cpt, xr, 0, lane, two, acc);
        const int row0 = (sub * rb_tiles + (warp * spw + l) * tps + t) * 16;
        const int lrow0 = ((warp * spw + l) * tps + t) * 16;   // within the unit
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int tl = frag_tok(lane, nt, r);
            if (tl < np) {
              if constexpr (EP) {
                osm[tl * OS + lrow0 + frag_row(lane, r)] = __float2bfloat16_rn(acc[nt][r]);
              } else {
                const int pi = ch * GR_CHUNK + tl;
                int tok, slot;
                if (pb < 0) { tok = pi; slot = a.k; }
                else { tok = rv.pair_tok[pb + pi]; slot = rv.pair_slot[pb + pi]; }
                a.part[(static_cast<int64_t>(tok) * (a.k + 1) + slot) * H + row0 + frag_row(lane, r)] = acc[nt][r];
              }
            }
          }
      }
      __syncwarp();
      if (lane == 0 && q + XT_NST < Q) ring.issue(q + XT_NST, src(q + XT_NST), sbytes);
    }
    if constexpr (EP) {
      // the unit's rows to their sources: row tl of the unit is the received row
      // pair_tok[pb + ch * 16 + tl] (no shared slot on the receiving side); each source's
      // counter takes one release add per row piece, after the CTA barrier that follows
      // the piece's stores
      __syncthreads();
      const int vec = rb_tiles * 16 / 8;   // 16-byte vectors per output row
      for (int i = threadIdx.x; i < np * vec; i += blockDim.x) {
        const int tl = i / vec, c = (i % vec) * 8;
        const int r = rv.pair_tok[pb + ch * GR_CHUNK + tl];
        const int srcr = r / ep.cap;
        const int pair = __ldcg(ep_win(ep.window, ep.G, ep.cap, H).meta + r) >> 9;
        __nv_bfloat16* to = ep_win(reinterpret_cast<const void*>(ep.peers[srcr]), ep.G, ep.cap, H).back +
                            static_cast<int64_t>(pair) * H + sub * rb_tiles * 16 + c;
        *reinterpret_cast<uint4*>(to) = *reinterpret_cast<const uint4*>(osm + tl * OS + c);
      }
      __syncthreads();
      if (threadIdx.x < np) {
        const int r = rv.pair_tok[pb + ch * GR_CHUNK + threadIdx.x];
        red_release_sys(ep_win(reinterpret_cast<const void*>(ep.peers[r / ep.cap]), ep.G, ep.cap, H).ccnt + ep.rank,
                        1ull);
      }
    }
  }
  cp_async_wait<0>();
}

// ------------------------------------------------------------------ dense experts (tcgen05)
// An expert that receives at least XtArgs::dense_min tokens is a real contraction: its
// gate/up and down run on the 5th-generation tensor cores instead of the grouped
// mma.sync kernels (which then skip it).  Item = (slot, token tile of up to TC_N pairs,
// row block of 128 weight rows), K in groups of 128 (one quantisation group).
//
// Per group the CTA copies, asynchronously and two groups ahead (cp.async, a ring of
// TC_ST stages), the row block's raw W4 chunks (8 stream tiles x 1056 bytes) and the
// tile's activation rows straight into the canonical K-major operand layout
// (umma.cuh); it expands the int4 values in shared memory to 16-bit integers q = u - 8
// (exact in bf16 and fp16), and one thread issues the group's eight K = 16 tcgen05.mma
// steps into a fresh fp32 accumulator in tensor memory (M = 128 weight rows, N = the
// tile's pairs rounded up to 16; two accumulators alternate).  While the tensor core
// works on group g, every thread reads group g - 1's accumulator (tcgen05.ld) and adds
// it, times its row's bf16 scale, into fp32 registers: the per-group partial sums and
// scaling of the grouped kernels, so both paths round alike (one accumulator chained
// over all of K lost low bits in the tensor core's fp32 additions).  Gate/up multiplies
// bf16 q by the bf16 activations as stored; down multiplies fp16 q by the fp16 h rows.
// All waits are bounded.  Epilogue: gate/up rows of one intermediate column meet through
// shared memory for SiLU(gate) * up in the reference's rounding order; down writes the
// fp32 expert output rows the combine reads.
constexpr int TC_THREADS = 512;
constexpr int TC_COLS = TC_N / (TC_THREADS / 128);   // accumulator columns per thread
constexpr int TC_ROWS_PT = TC_N * 16 / TC_THREADS;   // activation rows a thread copies per group
constexpr int TC_KS = 128;                      // K per stage (one quantisation group)
constexpr int TC_ST = 3;                        // ring stages
constexpr int TC_CHB = 8 * TC_KS + 32;          // one stream tile's group chunk (nibbles + scales)
constexpr int TC_A_BYTES = 128 * TC_KS * 2;     // 128 weight rows x 128 K, 16-bit
constexpr int TC_B_BYTES = TC_N * TC_KS * 2;    // TC_N rows x 128 K, 16-bit
constexpr int TC_RAW_BYTES = 8 * TC_CHB;        // the row block's 8 raw chunks
constexpr int TC_STAGE_BYTES = TC_A_BYTES + TC_B_BYTES + TC_RAW_BYTES;
constexpr int TC_HEAD = 1024 + (static_cast<int>(sizeof(GrTable)) + 1023) / 1024 * 1024;
constexpr size_t TC_SMEM = TC_HEAD + static_cast<size_t>(TC_ST) * TC_STAGE_BYTES;
constexpr uint32_t TC_TMEM_COLS = 2 * TC_N;     // two accumulators
static_assert(TC_SMEM <= 227 * 1024, "tcgen05 expert stages exceed shared memory");
static_assert(TC_STAGE_BYTES % 128 == 0 && TC_CHB % 16 == 0, "stage alignment");

// Byte offset of (row, K octet) in a canonical K-major tile of TC_KS columns.
__device__ __forceinline__ int tc_off(int row, int octet) {
  return ((row >> 3) * (TC_KS / 8) + octet) * 128 + (row & 7) * 16;
}

// Expand one W4 task of a raw chunk (16 bytes of nibbles: lane `ln`'s steps 4v .. 4v + 3)
// to the 16-bit integers q = u - 8 of A-tile rows row0 + gid and row0 + gid + 8.
// (MAGIC | u is 128 + u in bf16 or 1024 + u in fp16; subtracting OFF = MAGIC + 8 is exact.)
template <bool BF16>
__device__ __forceinline__ void tc_expand_task(uint8_t* As, const uint8_t* chunk, int v, int ln, int row0) {
  const uint4 wv = *reinterpret_cast<const uint4*>(chunk + v * 512 + ln * 16);
  const int gid = ln >> 2, tig = ln & 3;
  constexpr uint32_t MAGIC = BF16 ? 0x43004300u : 0x64006400u;
  const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int p = 0; p < 2; ++p) {           // steps (4v + 2p, 4v + 2p + 1): K octet 8v + 4p + tig
    const int octet = 8 * v + 4 * p + tig;
#pragma unroll
    for (int h = 0; h < 2; ++h) {         // row gid (nibbles 0, 2, 4, 6) or gid + 8 (1, 3, 5, 7)
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint32_t x = w[2 * p + e] >> (4 * h);
        uint32_t c[2] = {lop3_and_or(x, 0x000F000Fu, MAGIC), lop3_and_or(x >> 8, 0x000F000Fu, MAGIC)};
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          if constexpr (BF16) {
            const __nv_bfloat162 q = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&c[j]),
                                             __bfloat162bfloat162(__ushort_as_bfloat16(0x4308)));
            o[2 * e + j] = *reinterpret_cast<const uint32_t*>(&q);
          } else {
            const __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&c[j]),
                                      __half2half2(__ushort_as_half(0x6408)));
            o[2 * e + j] = *reinterpret_cast<const uint32_t*>(&q);
          }
        }
      }
      *reinterpret_cast<uint4*>(As + tc_off(row0 + gid + 8 * h, octet)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// The item's slot, token tile and row block (table built with TC_N-pair chunks).
template <typename ET>
__device__ __forceinline__ void tc_item(const GrTable& tb, const MoeArgs<ET>& a, const RouteView& rv, int item,
                                        int per, bool up, int& slot, int& tt, int& rb, const uint8_t*& w, int& np,
                                        int& pbase) {
  slot = gr_slot_of(tb, item);
  const int r = item - tb.first[slot];
  tt = r / per;
  rb = r % per;
  np = min(TC_N, gr_pairs(a, rv, slot) - tt * TC_N);
  if (a.has_shared && slot == 0) {
    w = up ? a.sgu : a.sdn;
    pbase = -1;
  } else {
    const int ai = slot - a.has_shared;
    const int e = rv.active[ai];
    w = up ? a.gu + e * a.gu_stride : a.dn + e * a.dn_stride;
    pbase = rv.pair_off[ai];
  }
}

struct TcRing {
  uint8_t* stages;
  uint64_t* full;     // 2 barriers: accumulator (g % 2) holds group g
  uint32_t tmem;
  int g;              // groups issued so far (all items of the CTA)
};

// What one item streams: 8 stream tiles (tile0 .. + 3 -> A rows 0-63, tile1 .. + 3 ->
// rows 64-127) of a K-wide W4 matrix, and the activation rows src[rows[i]] (16-bit,
// row stride src_ld elements) of the tile's pairs [0, np), zero up to nn.
struct TcOperands {
  const uint8_t* w;
  int tile0, tile1, K;
  const uint8_t* src;
  int64_t src_ld;
  int np, nn;
};

__device__ __forceinline__ uint8_t* tc_stage(const TcRing& r, int g) { return r.stages + (g % TC_ST) * TC_STAGE_BYTES; }

// Copy task i of this thread: activation row n and K octet of the B tile.  Task t =
// i * TC_THREADS + threadIdx.x covers row group t / 128, octets 4 ((t / 32) % 4) ..
// + 3 (lane / 8) of rows (lane % 8).
__device__ __forceinline__ void tc_copy_slot(int i, int& n, int& octet) {
  const int t = i * TC_THREADS + threadIdx.x, lane = t & 31;
  n = (t >> 7) * 8 + (lane & 7);
  octet = ((t >> 5) & 3) * 4 + (lane >> 3);
}

// Every thread: its cp.async copies of group kg into stage g (one commit group).
__device__ __forceinline__ void tc_load(const TcRing& r, const TcOperands& o, const int (&rows)[TC_ROWS_PT], int g,
                                        int kg) {
  uint8_t* st = tc_stage(r, g);
  uint8_t* Bs = st + TC_A_BYTES;
  uint8_t* raw = Bs + TC_B_BYTES;
  for (int i = threadIdx.x; i < 8 * (TC_CHB / 16); i += TC_THREADS) {
    const int t8 = i / (TC_CHB / 16), c = i % (TC_CHB / 16);
    const int tile = t8 < 4 ? o.tile0 + t8 : o.tile1 + (t8 - 4);
    cp_async16(raw + t8 * TC_CHB + c * 16,
               o.w + W4Fmt<128>::tile_offset(tile, o.K, 0) + static_cast<int64_t>(kg) * TC_CHB + c * 16, true);
  }
  // a warp fills four whole core matrices (8 rows x 4 K octets, 512 contiguous bytes)
#pragma unroll
  for (int i = 0; i < TC_ROWS_PT; ++i) {
    int n, octet;
    tc_copy_slot(i, n, octet);
    if (n < o.nn)
      cp_async16(Bs + tc_off(n, octet), o.src + (static_cast<int64_t>(rows[i]) * o.src_ld + kg * TC_KS + octet * 8) * 2,
                 n < o.np);
  }
  cp_async_commit();
}

// Group kg (in stage g = r.g, copies landed): expand A, then one thread issues the MMAs
// into accumulator g % 2 and commits them to full[g % 2].
template <bool BF16>
__device__ __forceinline__ void tc_issue(TcRing& r, uint32_t idesc) {
  uint8_t* As = tc_stage(r, r.g);
  const uint8_t* raw = As + TC_A_BYTES + TC_B_BYTES;
#pragma unroll
  for (int i = 0; i < 512 / TC_THREADS; ++i) {   // 8 raw chunks x 64 tasks of 16 bytes
    const int task = threadIdx.x + i * TC_THREADS;
    const int t8 = task >> 6, v = (task >> 5) & 1, ln = task & 31;
    tc_expand_task<BF16>(As, raw + t8 * TC_CHB, v, ln, t8 * 16);
  }
  fence_proxy_async();   // the generic-proxy stores (and landed copies) before the tensor core reads them
  __syncthreads();
  if (threadIdx.x == 0) {
    umma::fence_after_sync();
    const uint32_t a0 = smem_u32(As), b0 = a0 + TC_A_BYTES;
    const uint32_t d = r.tmem + (r.g & 1) * TC_N;
#pragma unroll
    for (int s = 0; s < TC_KS / 16; ++s)
      umma::mma_f16(d, umma::smem_desc(a0 + s * 256, 128, (TC_KS / 8) * 128),
                    umma::smem_desc(b0 + s * 256, 128, (TC_KS / 8) * 128), idesc, s > 0);
    umma::commit(r.full + (r.g & 1));
  }
  ++r.g;
}

// Every thread: wait (bounded) for group g's accumulator and add its columns
// [c0, c0 + TC_COLS) of this warp's 32 rows, times the row's scale (from the group's raw
// chunk), into acc.
__device__ __forceinline__ bool tc_accumulate(const TcRing& r, const XtArgs& args, int g, int c0, int nn, int row,
                                              float (&acc)[TC_COLS]) {
  const bool ok = __syncthreads_and(mbar_wait(r.full + (g & 1), (g >> 1) & 1, args.status, args.limit));
  if (!ok) return false;
  umma::fence_after_sync();
  const uint8_t* raw = tc_stage(r, g) + TC_A_BYTES + TC_B_BYTES;
  const int rr = row & 15;   // scale position 2 gid + h <-> row gid + 8 h of the tile
  const float scale = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(
      raw + (row >> 4) * TC_CHB + 8 * TC_KS + 2 * (2 * (rr & 7) + (rr >> 3))));
  const int q = (threadIdx.x >> 5) & 3;
  const uint32_t base = r.tmem + (static_cast<uint32_t>(32 * q) << 16) + (g & 1) * TC_N + c0;
#pragma unroll
  for (int c = 0; c < TC_COLS / 16; ++c) {
    if (c0 + 16 * c < nn) {
      float v[16];
      umma::ld16(base + 16 * c, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[16 * c + j] = fmaf(scale, v[j], acc[16 * c + j]);
    }
  }
  umma::fence_before_sync();
  __syncthreads();   // every thread is done with the group's stage and accumulator
  return true;
}

// All groups of one item; acc = this thread's TC_COLS fp32 sums (row 32 (warp % 4) +
// lane, columns TC_COLS (warp / 4) ..).  False when a bounded wait expired.
template <bool BF16>
__device__ __forceinline__ bool tc_item_run(TcRing& r, const XtArgs& args, const TcOperands& o, int ngroups,
                                            const int (&rows)[TC_ROWS_PT], float (&acc)[TC_COLS]) {
  const uint32_t idesc = umma::idesc_16(128, o.nn, BF16);
  const int row = 32 * ((threadIdx.x >> 5) & 3) + (threadIdx.x & 31);
  const int c0 = TC_COLS * (threadIdx.x >> 7);
#pragma unroll
  for (int j = 0; j < TC_COLS; ++j) acc[j] = 0.f;
  const int g0 = r.g;
  tc_load(r, o, rows, g0, 0);
  if (ngroups > 1) tc_load(r, o, rows, g0 + 1, 1); else cp_async_commit();
  for (int kg = 0; kg < ngroups; ++kg) {
    cp_async_wait<1>();    // this thread's copies of group kg landed
    __syncthreads();       // everyone's
    tc_issue<BF16>(r, idesc);
    if (kg > 0 && !tc_accumulate(r, args, r.g - 2, c0, o.nn, row, acc)) return false;
    // stage of group kg - 1 is free (its MMAs completed): copies of group kg + 2
    if (kg + 2 < ngroups) tc_load(r, o, rows, g0 + kg + 2, kg + 2); else cp_async_commit();
  }
  cp_async_wait<0>();
  return tc_accumulate(r, args, r.g - 1, c0, o.nn, row, acc);
}

// Setup common to both kernels: barriers, the tensor-memory allocation (warp 0).
__device__ __forceinline__ void tc_setup(uint8_t* smem, TcRing& r) {
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint32_t* tbase = reinterpret_cast<uint32_t*>(smem + 256);
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) mbar_init(bars + i, 1);
  }
  fence_barrier_init();
  if (threadIdx.x < 32) umma::tmem_alloc(tbase, TC_TMEM_COLS);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  r.stages = smem + TC_HEAD;
  r.full = bars;
  r.tmem = *tbase;
  r.g = 0;
}

// Teardown: every MMA this CTA issued has completed (or a bounded wait gave up, after
// which the last group's commit is waited for once more, bounded, and the copies in
// flight drained), then warp 0 frees the columns.
__device__ __forceinline__ void tc_teardown(TcRing& r, const XtArgs& args, bool ok) {
  if (!ok && r.g > 0) {
    const int last = r.g - 1;
    const long long t0 = clock64();
    while (!mbar_try_wait(r.full + (last & 1), (last >> 1) & 1))
      if (clock64() - t0 > args.limit) break;
  }
  cp_async_wait<0>();
  umma::fence_before_sync();
  __syncthreads();
  if (threadIdx.x < 32) {
    umma::fence_after_sync();
    umma::tmem_free(r.tmem, TC_TMEM_COLS);
  }
}

// Gate/up of the dense slots.  Row block rb = intermediate columns [64 rb, 64 rb + 64):
// A rows 0-63 are their gate rows (stream tiles 4 rb ..), rows 64-127 their up rows
// (tiles I / 16 + 4 rb ..); h = round(round(SiLU(round(gate))) * round(up)) per pair,
// stored as fp16 like the grouped kernel's.
__global__ void __launch_bounds__(TC_THREADS, 1) moe_up_tc_kernel(XtArgs args) {
  const MoeArgs<__nv_bfloat16>& a = args.m;
  extern __shared__ __align__(16) uint8_t smem[];
  GrTable& tb = *reinterpret_cast<GrTable*>(smem + 1024);
  const RouteView rv = route_view(a.ws, a.T, a.E, a.k);
  const int H = a.H, I = a.I, per = I / 64;
  pdl_wait();   // the lists come from the predecessor
  pdl_trigger();
  gr_build_table(tb, a, rv, per, args.dense_min, true, TC_N);
  if (blockIdx.x >= tb.total) return;
  TcRing r;
  tc_setup(smem, r);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3, row = 32 * q + lane, c0 = TC_COLS * (warp >> 2);
  bool ok = true;
  for (int it = blockIdx.x; it < tb.total && ok; it += gridDim.x) {
    int sl, tt, rb, np, pb;
    const uint8_t* w;
    tc_item(tb, a, rv, it, per, true, sl, tt, rb, w, np, pb);
    int rows[TC_ROWS_PT];
#pragma unroll
    for (int i = 0; i < TC_ROWS_PT; ++i) {
      int n, octet;
      tc_copy_slot(i, n, octet);
      n = min(n, np - 1);
      rows[i] = pb < 0 ? tt * TC_N + n : rv.pair_tok[pb + tt * TC_N + n];
    }
    const TcOperands o{w, 4 * rb, I / 16 + 4 * rb, H, reinterpret_cast<const uint8_t*>(a.x), H, np,
                       (np + 15) & ~15};
    float acc[TC_COLS];
    ok = tc_item_run<true>(r, args, o, H / TC_KS, rows, acc);
    if (!ok) break;
    // the up rows (quarters 2, 3) go through the first stage (idle: every MMA and copy is done)
    float* ubuf = reinterpret_cast<float*>(r.stages);   // [64][TC_N + 1]
    if (q >= 2) {
#pragma unroll
      for (int j = 0; j < TC_COLS; ++j)
        if (c0 + j < o.nn) ubuf[(row - 64) * (TC_N + 1) + c0 + j] = rbf(acc[j]);
    }
    __syncthreads();
    if (q < 2) {
#pragma unroll
      for (int j = 0; j < TC_COLS; ++j) {
        const int n = c0 + j;
        if (n < np) {
          const float gr = rbf(acc[j]), ur = ubuf[row * (TC_N + 1) + n];
          const float h = rbf(rbf(silu_f(gr)) * ur);
          const int pi = tt * TC_N + n;
          const int64_t hrow = pb < 0 ? static_cast<int64_t>(a.T) * a.k + pi : pb + pi;
          reinterpret_cast<__half*>(a.hbuf)[hrow * I + rb * 64 + row] = __float2half_rn(h);
        }
      }
    }
    __syncthreads();   // ubuf free for the next item's stages
  }
  tc_teardown(r, args, ok);
}

// Down of the dense slots.  Row block rb = output columns [128 rb, 128 rb + 128) (stream
// tiles 8 rb ..); K = I from the fp16 h rows; fp32 outputs to part[token][slot].
__global__ void __launch_bounds__(TC_THREADS, 1) moe_down_tc_kernel(XtArgs args) {
  const MoeArgs<__nv_bfloat16>& a = args.m;
  extern __shared__ __align__(16) uint8_t smem[];
  GrTable& tb = *reinterpret_cast<GrTable*>(smem + 1024);
  const RouteView rv = route_view(a.ws, a.T, a.E, a.k);
  const int H = a.H, I = a.I, per = H / 128;
  pdl_wait();   // h comes from the predecessors (gate/up)
  pdl_trigger();
  gr_build_table(tb, a, rv, per, args.dense_min, true, TC_N);
  if (blockIdx.x >= tb.total) return;
  TcRing r;
  tc_setup(smem, r);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = 32 * (warp & 3) + lane, c0 = TC_COLS * (warp >> 2);
  bool ok = true;
  for (int it = blockIdx.x; it < tb.total && ok; it += gridDim.x) {
    int sl, tt, rb, np, pb;
    const uint8_t* w;
    tc_item(tb, a, rv, it, per, false, sl, tt, rb, w, np, pb);
    const int64_t hb = (pb < 0 ? static_cast<int64_t>(a.T) * a.k : pb) + tt * TC_N;
    int rows[TC_ROWS_PT];
#pragma unroll
    for (int i = 0; i < TC_ROWS_PT; ++i) {
      int n, octet;
      tc_copy_slot(i, n, octet);
      rows[i] = static_cast<int>(hb) + min(n, np - 1);
    }
    const TcOperands o{w, 8 * rb, 8 * rb + 4, I, reinterpret_cast<const uint8_t*>(a.hbuf), I, np, (np + 15) & ~15};
    float acc[TC_COLS];
    ok = tc_item_run<false>(r, args, o, I / TC_KS, rows, acc);
    if (!ok) break;
#pragma unroll
    for (int j = 0; j < TC_COLS; ++j) {
      const int n = c0 + j;
      if (n < np) {
        const int pi = tt * TC_N + n;
        int tok, slot;
        if (pb < 0) { tok = pi; slot = a.k; }
        else { tok = rv.pair_tok[pb + pi]; slot = rv.pair_slot[pb + pi]; }
        a.part[(static_cast<int64_t>(tok) * (a.k + 1) + slot) * H + rb * 128 + row] = acc[j];
      }
    }
  }
  tc_teardown(r, args, ok);
}

// Combine (fused/model.py:296-307 with fused_ops.py:165-172): per token, the routed
// experts in ascending id, each raw output rounded to the activation dtype, times its
// weight (rounded), added with a rounding; then + round(round(shared) * gate) when a
// shared expert is present; then, in residual mode, out = round(out + moe) in place.
template <typename ET>
__global__ void moe_combine_kernel(const float* __restrict__ part, void* ws, ET* __restrict__ out,
                                   int T, int H, int E, int k, int has_shared, int residual) {
  const RouteView rv = route_view(ws, T, E, k);
  const int t = blockIdx.x;
  int order[32];
  for (int j = 0; j < k; ++j) order[j] = j;
  for (int i = 1; i < k; ++i)
    for (int j = i; j > 0 && rv.topk_idx[t * k + order[j]] < rv.topk_idx[t * k + order[j - 1]]; --j) {
      int tmp = order[j]; order[j] = order[j - 1]; order[j - 1] = tmp;
    }
  const float sg = has_shared ? rv.shared_gate[t] : 0.f;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < k; ++j) {
      const int s = order[j];
      const float y = rnd<ET>(part[(static_cast<int64_t>(t) * (k + 1) + s) * H + c]);
      acc = rnd<ET>(acc + rnd<ET>(y * rv.topk_w[t * k + s]));
    }
    if (has_shared) {
      const float y = rnd<ET>(part[(static_cast<int64_t>(t) * (k + 1) + k) * H + c]);
      acc = rnd<ET>(acc + rnd<ET>(y * sg));
    }
    ET* o = out + static_cast<int64_t>(t) * H + c;
    *o = from_f<ET>(residual ? to_f(*o) + acc : acc);
  }
}

// Combine fused with the next RMSNorm (the boundary between decoder layers): per token
// t, hidden[t] = bf16(hidden[t] + moe(t)) with moe(t) summed as moe_combine_kernel does
// (ascending expert, rounding at each add, then the gated shared expert), then
// normed[t] = bf16(bf16(h * rsqrt(mean(h^2) + eps)) * bf16(gamma + 1)) as
// residual_norm_kernel, and the optional feature tap (h, or the normed row).
// A cluster of CN_SPLIT CTAs per token (64 SMs at T = 16 instead of 16: one CTA per
// token kept only 16 SMs' worth of loads in flight); thread g = rank * CN_THREADS + tid of
// the token's cluster owns runs of 4 columns (16-byte loads of the fp32 expert outputs,
// all k + 1 slots of a run issued before the ordered sum).  The sum of squares is reduced
// as block_sum reduces one CN_TOTAL-thread block -- each warp's tree, then one tree over
// the warp sums in warp order, gathered from the cluster through distributed shared
// memory -- so the norm has the bits of a one-CTA-per-token kernel.
constexpr int CN_THREADS = 128;
constexpr int CN_SPLIT = 4;
constexpr int CN_TOTAL = CN_THREADS * CN_SPLIT;
static_assert(CN_TOTAL / 32 <= 32, "the warp sums of a token fit one warp");

// Expert-parallel form (ep.window set): the expert outputs are the bf16 rows the expert
// owners stored into this rank's window (routed pair p = t k + s at back row p, the
// shared expert's at row T k + t) -- the values the f32 path rounds to bf16 first, so the
// sums have the same bits; every CTA waits (bounded) for every rank's combine flag
// first, and the last CTA closes the exchange.
struct EpRecv {
  void* window;   // null: the f32 outputs of the workspace
  int G, cap;
};

template <int KMAX>
__global__ void __launch_bounds__(CN_THREADS) moe_combine_norm_kernel(
    const float* __restrict__ part, void* ws, __nv_bfloat16* __restrict__ hidden, int T, int H, int E, int k,
    int has_shared, const __nv_bfloat16* __restrict__ gamma, __nv_bfloat16* __restrict__ normed, float eps,
    __nv_bfloat16* __restrict__ tap, int64_t ldf, int tap_normed, EpRecv ep) {
  __shared__ int s_slot[KMAX];
  __shared__ float s_w[KMAX];
  __shared__ float red[CN_TOTAL / 32];
  cluster_arrive_relaxed();   // the peers' shared memory is written only after every CTA started
  const int rank = blockIdx.x % CN_SPLIT;
  const int g = rank * CN_THREADS + threadIdx.x;   // thread index within the token's cluster
  // before the wait: everything but the expert outputs -- the routing (from the route
  // kernel), the residual row (from the mixer's projection) and the norm weight are
  // older than the predecessor (the down projection)
  const RouteView rv = route_view(ws, T, E, k);
  const int t = blockIdx.x / CN_SPLIT;
  if (threadIdx.x < k) {
    const int e = rv.topk_idx[t * k + threadIdx.x];
    int rank = 0;
    for (int j = 0; j < k; ++j) rank += rv.topk_idx[t * k + j] < e;
    s_slot[rank] = threadIdx.x;
    s_w[rank] = rv.topk_w[t * k + threadIdx.x];
  }
  const float sg = has_shared ? rv.shared_gate[t] : 0.f;
  __nv_bfloat16* h = hidden + static_cast<int64_t>(t) * H;
  const bool one = H <= 4 * CN_TOTAL;   // each thread at most one 4-column chunk
  uint2 h0 = make_uint2(0u, 0u), g0 = make_uint2(0u, 0u), n0 = make_uint2(0u, 0u);
  if (one && 4 * g < H) {
    h0 = *reinterpret_cast<const uint2*>(h + 4 * g);
    g0 = *reinterpret_cast<const uint2*>(gamma + 4 * g);
  }
  pdl_wait();
  pdl_trigger();
  __shared__ int s_epoch;
  EpWin me{};
  if (ep.window) {
    me = ep_win(ep.window, ep.G, ep.cap, H);
    if (threadIdx.x == 0) s_epoch = me.hdr[0] + 1;
    __syncthreads();
    if (threadIdx.x < ep.G) ep_wait_count(me.ccnt + threadIdx.x, s_epoch * EP_ROUND, me.hdr);
  }
  __syncthreads();
  const float* pt = part + static_cast<int64_t>(t) * (k + 1) * H;
  float ss = 0.f;
  auto back4 = [&](int64_t row, int c) {
    const uint2 u = __ldcg(reinterpret_cast<const uint2*>(me.back + row * H + c));
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
  };
  for (int c = 4 * g; c < H; c += 4 * CN_TOTAL) {
    float4 y[KMAX + 1];
    if (ep.window) {
#pragma unroll
      for (int j = 0; j < KMAX; ++j)
        if (j < k) y[j] = back4(static_cast<int64_t>(t) * k + s_slot[j], c);
      if (has_shared) y[KMAX] = back4(static_cast<int64_t>(T) * k + t, c);
    } else {
#pragma unroll
      for (int j = 0; j < KMAX; ++j)
        if (j < k) y[j] = *reinterpret_cast<const float4*>(pt + static_cast<int64_t>(s_slot[j]) * H + c);
      if (has_shared) y[KMAX] = *reinterpret_cast<const float4*>(pt + static_cast<int64_t>(k) * H + c);
    }
    const uint2 hraw = one ? h0 : *reinterpret_cast<const uint2*>(h + c);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      if (j < k) {
        const float w = s_w[j];
        acc[0] = rbf(acc[0] + rbf(rbf(y[j].x) * w));
        acc[1] = rbf(acc[1] + rbf(rbf(y[j].y) * w));
        acc[2] = rbf(acc[2] + rbf(rbf(y[j].z) * w));
        acc[3] = rbf(acc[3] + rbf(rbf(y[j].w) * w));
      }
    }
    if (has_shared) {
      acc[0] = rbf(acc[0] + rbf(rbf(y[KMAX].x) * sg));
      acc[1] = rbf(acc[1] + rbf(rbf(y[KMAX].y) * sg));
      acc[2] = rbf(acc[2] + rbf(rbf(y[KMAX].z) * sg));
      acc[3] = rbf(acc[3] + rbf(rbf(y[KMAX].w) * sg));
    }
    const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&hraw);
    const float2 h01 = __bfloat1622float2(hp[0]), h23 = __bfloat1622float2(hp[1]);
    const __nv_bfloat162 n01 = __floats2bfloat162_rn(h01.x + acc[0], h01.y + acc[1]);
    const __nv_bfloat162 n23 = __floats2bfloat162_rn(h23.x + acc[2], h23.y + acc[3]);
    uint2 out;
    out.x = *reinterpret_cast<const uint32_t*>(&n01);
    out.y = *reinterpret_cast<const uint32_t*>(&n23);
    *reinterpret_cast<uint2*>(h + c) = out;
    n0 = out;
    const float2 f01 = __bfloat1622float2(n01), f23 = __bfloat1622float2(n23);
    ss += f01.x * f01.x + f01.y * f01.y + f23.x * f23.x + f23.y * f23.y;
  }
  {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    ss = warp_sum(ss);
    cluster_wait();
    if (lane == 0) {
      cg::cluster_group cl = cg::this_cluster();
#pragma unroll
      for (int r = 0; r < CN_SPLIT; ++r) cl.map_shared_rank(red, r)[rank * (CN_THREADS / 32) + warp] = ss;
    }
    cg::this_cluster().sync();   // every warp sum has landed; no peer writes after this
    float tt = lane < CN_TOTAL / 32 ? red[lane] : 0.f;
    ss = warp_sum(tt);
  }
  const float inv = rsqrtf(ss / H + eps);
  for (int c = 4 * g; c < H; c += 4 * CN_TOTAL) {
    const uint2 hraw = one ? n0 : *reinterpret_cast<const uint2*>(h + c);
    const uint2 graw = one ? g0 : *reinterpret_cast<const uint2*>(gamma + c);
    const __nv_bfloat16* hv = reinterpret_cast<const __nv_bfloat16*>(&hraw);
    const __nv_bfloat16* gv = reinterpret_cast<const __nv_bfloat16*>(&graw);
    __nv_bfloat16 yv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float g = rbf(__bfloat162float(gv[i]) + 1.f);
      yv[i] = __float2bfloat16_rn(rbf(__bfloat162float(hv[i]) * inv) * g);
    }
    const uint2 yraw = *reinterpret_cast<const uint2*>(yv);
    *reinterpret_cast<uint2*>(normed + static_cast<int64_t>(t) * H + c) = yraw;
    if (tap) {
      // 8-byte stores need ldf and the tap column to be multiples of 4
      *reinterpret_cast<uint2*>(tap + static_cast<int64_t>(t) * ldf + c) = tap_normed ? yraw : hraw;
    }
  }
  if (ep.window && ep_last_cta(me.hdr + 3) && threadIdx.x == 0) me.hdr[0] = s_epoch;
}

// Router logits of the fused-ops operator: dense [E, H] weights, one warp per (t, e),
// fp32 accumulate, one rounding to the activation dtype.
template <typename ET>
__global__ void router_dense_kernel(const ET* __restrict__ x, const ET* __restrict__ w, ET* __restrict__ out,
                                    int T, int H, int E) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (gw >= T * E) return;
  const int t = gw / E, e = gw % E;
  float acc = 0.f;
  for (int c = lane; c < H; c += 32) acc = fmaf(to_f(x[static_cast<int64_t>(t) * H + c]), to_f(w[static_cast<int64_t>(e) * H + c]), acc);
  acc = warp_sum(acc);
  if (lane == 0) out[static_cast<int64_t>(t) * E + e] = from_f<ET>(acc);
}

// ------------------------------------------------------------------ host launchers
template <typename LT>
static int launch_route(const void* logits, int64_t ldl, int T, int E, int k, int shared_col,
                        int act_is_f16, void* ws, const void* x, int H, int G, cudaStream_t s, int tie_order = 1) {
  const size_t smem = ROUTE_TPB * route_warp_smem(E);
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    err = cudaFuncSetAttribute(route_topk_kernel<LT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
  });
  if (err != cudaSuccess) return cuda_status(err, "route smem attribute");
  if (smem > 64 * 1024) return fail(QW_ERR_UNSUPPORTED, "route: too many experts");
  QW_LAUNCH_PDL("moe route", route_topk_kernel<LT>, dim3((T + ROUTE_TPB - 1) / ROUTE_TPB), dim3(32 * ROUTE_TPB), smem,
                s, static_cast<const LT*>(logits), ldl, T, E, k, shared_col, act_is_f16, ws,
                static_cast<const __nv_bfloat16*>(x), H, G, tie_order);
  return QW_OK;
}

static int launch_route_lists(int T, int E, int k, int lo, int ne, void* ws, cudaStream_t s) {
  const size_t smem = (3 * static_cast<size_t>(E) + 64) * sizeof(int);
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    err = cudaFuncSetAttribute(route_lists_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
  });
  if (err != cudaSuccess) return cuda_status(err, "route lists smem attribute");
  QW_LAUNCH_PDL("moe route lists", route_lists_kernel, dim3(1), dim3(1024), smem, s, T, E, k, lo, ne, ws);
  return QW_OK;
}

template <class Fmt, int NT, int PF, class FmtUp = Fmt>
static int launch_experts_nt(const MoeArgs<typename Fmt::ET>& a, cudaStream_t s, bool up, bool down) {
  const int slots = 1 + (a.E < a.T * a.k ? a.E : a.T * a.k);
  if (up) {
    const int jb = (a.I / 16 + UP_JT - 1) / UP_JT;
    QW_LAUNCH_PDL("moe up", moe_up_kernel<FmtUp, NT, PF>, dim3(slots, jb), dim3(SG_WARPS * 32), 0, s, a);
  }
  if (down) {
    QW_LAUNCH_PDL("moe down", moe_down_kernel<Fmt, NT, PF>, dim3(slots, (a.H / 16 + SG_WARPS - 1) / SG_WARPS),
                  dim3(SG_WARPS * 32), 0, s, a);
  }
  return QW_OK;
}

// Activation tile width: 8 tokens when routed experts average at most ~2 tokens (the
// block-verify case: 16 tokens x top-8 over 256 experts), else 16.
template <class Fmt, int PF, class FmtUp = Fmt>
static int launch_experts(const MoeArgs<typename Fmt::ET>& a, cudaStream_t s, bool up, bool down) {
  const int64_t pairs = a.pairs_hint > 0 ? a.pairs_hint : static_cast<int64_t>(a.T) * a.k;
  if (pairs <= 2LL * a.E) return launch_experts_nt<Fmt, 1, PF, FmtUp>(a, s, up, down);
  return launch_experts_nt<Fmt, 2, PF, FmtUp>(a, s, up, down);
}

static int sm_count() {
  static int counts[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!counts[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

constexpr size_t XT_SMEM_LIMIT = 227 * 1024;



// Shapes the bulk-copy kernels take: the verify block (T <= 16), and stage geometry
// that tiles the weights exactly.
struct XtPlan {
  bool up_ok, down_ok;
  int down_tps, down_spw;
  size_t up_smem, down_smem;
  size_t down_ep_smem;   // grouped down kernel with the expert-parallel send
};

template <int G>
static XtPlan xt_plan(const MoeArgs<__nv_bfloat16>& a) {
  XtPlan p{};
  constexpr int CHB = W4Fmt<G>::CHB;
  const bool small = a.T <= XT_MAXT && static_cast<int64_t>(a.T) * a.k <= XT_MAXT * 16 && a.H % 8 == 0 &&
                     (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.hbuf) & 15) == 0;
  const int nch = a.H / G;
  const int cps = nch < XT_UP_CPS ? nch : XT_UP_CPS;
  p.up_smem = xt_head_bytes(a.E) + (static_cast<size_t>(a.T) * (a.H + XT_PAD) * 2 + 127) / 128 * 128 +
              (static_cast<size_t>(a.T) * nch * 4 + 127) / 128 * 128 + static_cast<size_t>(XT_UP_WARPS) * XT_NST * cps * CHB;
  p.up_ok = small && nch % cps == 0 && cps % 2 == 0 && p.up_smem <= XT_SMEM_LIMIT;
  const int cpt = a.I / G;
  p.down_ok = false;
  if (small && cpt >= 1 && cpt <= XT_DN_CPS && XT_DN_CPS % cpt == 0) {
    p.down_tps = XT_DN_CPS / cpt;
    const int tiles = a.H / 16;
    p.down_spw = 0;
    for (int spw = 2; spw >= 1; --spw)
      if (tiles % (XT_DN_WARPS * spw * p.down_tps) == 0) { p.down_spw = spw; break; }
    p.down_smem = xt_head_bytes(a.E) + 3 * ((static_cast<size_t>(XT_MAXT) * (a.I + XT_PAD) * 2 + 127) / 128 * 128) +
                  static_cast<size_t>(XT_DN_WARPS) * XT_NST * p.down_tps * cpt * CHB;
    p.down_ok = p.down_spw > 0 && p.down_smem <= XT_SMEM_LIMIT;
  }
  return p;
}

template <int G>
static int launch_experts_bulk(const MoeArgs<__nv_bfloat16>& a, const XtPlan& p, cudaStream_t s, bool up,
                               bool down, int32_t* status) {
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    err = cudaFuncSetAttribute(moe_up_bulk_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(XT_SMEM_LIMIT));
    if (err == cudaSuccess)
      err = cudaFuncSetAttribute(moe_down_bulk_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(XT_SMEM_LIMIT));
  });
  if (err != cudaSuccess) return cuda_status(err, "moe bulk smem attribute");
  const WaitInjection inj = wait_injection();
  XtArgs xa{a, status, inj.limit > 0 ? inj.limit : QW_WAIT_LIMIT, 0};
  const int grid = sm_count();
  if (up) {
    QW_LAUNCH_PDL("moe up (bulk)", moe_up_bulk_kernel<G>, dim3(grid), dim3(XT_UP_WARPS * 32), p.up_smem, s, xa);
  }
  if (down) {
    QW_LAUNCH_PDL("moe down (bulk)", moe_down_bulk_kernel<G>, dim3(grid), dim3(XT_DN_WARPS * 32), p.down_smem, s, xa,
                  p.down_tps, p.down_spw);
  }
  return QW_OK;
}

// Shapes the grouped kernels take: I / 16 a multiple of the gate/up warp count and the
// bulk down kernel's stage geometry.
template <int G>
static bool grouped_plan(const MoeArgs<__nv_bfloat16>& a, XtPlan& p) {
  constexpr int CHB = W4Fmt<G>::CHB;
  const int nch = a.H / G;
  const int cps = nch < XT_UP_CPS ? nch : XT_UP_CPS;
  if ((a.I / 16) % XT_UP_WARPS || a.H % 8 || nch % cps || cps % 2 || (reinterpret_cast<uintptr_t>(a.x) & 15) ||
      (reinterpret_cast<uintptr_t>(a.hbuf) & 15) || a.has_shared + a.e_cnt > GR_MAX_SLOTS)
    return false;
  const size_t head = XT_BAR_BYTES + (sizeof(GrTable) + 127) / 128 * 128;
  p.up_smem = head + (static_cast<size_t>(GR_CHUNK) * (a.H + XT_PAD) * 2 + 127) / 128 * 128 +
              (static_cast<size_t>(GR_CHUNK) * nch * 4 + 127) / 128 * 128 +
              static_cast<size_t>(XT_UP_WARPS) * XT_NST * cps * CHB;
  const int cpt = a.I / G;
  if (cpt < 1 || cpt > XT_DN_CPS || XT_DN_CPS % cpt) return false;
  p.down_tps = XT_DN_CPS / cpt;
  const int tiles = a.H / 16;
  p.down_spw = 0;
  for (int spw = 2; spw >= 1; --spw)
    if (tiles % (XT_DN_WARPS * spw * p.down_tps) == 0) { p.down_spw = spw; break; }
  p.down_smem = head + 3 * ((static_cast<size_t>(GR_CHUNK) * (a.I + XT_PAD) * 2 + 127) / 128 * 128) +
                static_cast<size_t>(XT_DN_WARPS) * XT_NST * p.down_tps * cpt * CHB;
  if (p.down_spw > 0) {   // room for the expert-parallel output tile
    const int rb = XT_DN_WARPS * p.down_spw * p.down_tps * 16;
    p.down_ep_smem = p.down_smem + (static_cast<size_t>(GR_CHUNK) * (rb + 8) * 2 + 127) / 128 * 128;
  }
  return p.down_spw > 0 && p.up_smem <= GR_SMEM_LIMIT && p.down_smem <= GR_SMEM_LIMIT;
}

// Tokens per expert from which a routed expert runs on the tcgen05 kernels (0: never,
// the default: measured no faster than the grouped kernels on the benchmark's routings);
// see qw_moe_dense_threshold.
static std::atomic<int> g_dense_min{0};

// The dense path's shape limits: group 128 (one quantisation group per K stage), K and
// the row blocks whole, 16-byte aligned activation rows.
template <int G>
static int dense_min_for(const MoeArgs<__nv_bfloat16>& a, const EpSend* ep) {
  if (G != 128 || ep || a.H % 128 || a.I % 128 || (reinterpret_cast<uintptr_t>(a.x) & 15)) return 0;
  return g_dense_min.load(std::memory_order_relaxed);
}

template <int G>
static int launch_experts_grouped(const MoeArgs<__nv_bfloat16>& a, const XtPlan& p, cudaStream_t s, bool up,
                                  bool down, int32_t* status, const EpSend* ep = nullptr) {
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    err = cudaFuncSetAttribute(moe_up_grouped_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(GR_SMEM_LIMIT));
    if (err == cudaSuccess)
      err = cudaFuncSetAttribute(moe_down_grouped_kernel<G, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(GR_SMEM_LIMIT));
    if (err == cudaSuccess)
      err = cudaFuncSetAttribute(moe_down_grouped_kernel<G, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(GR_SMEM_LIMIT));
  });
  if (err != cudaSuccess) return cuda_status(err, "moe grouped smem attribute");
  const int dmin = dense_min_for<G>(a, ep);
  if (dmin > 0) {
    static std::once_flag once_tc;
    static cudaError_t err_tc = cudaSuccess;
    std::call_once(once_tc, [] {
      err_tc = cudaFuncSetAttribute(moe_up_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(TC_SMEM));
      if (err_tc == cudaSuccess)
        err_tc = cudaFuncSetAttribute(moe_down_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(TC_SMEM));
    });
    if (err_tc != cudaSuccess) return cuda_status(err_tc, "moe dense smem attribute");
  }
  const WaitInjection inj = wait_injection();
  XtArgs xa{a, status, inj.limit > 0 ? inj.limit : QW_WAIT_LIMIT, dmin};
  const int grid = sm_count();
  if (up) {
    QW_LAUNCH_PDL("moe up (grouped)", moe_up_grouped_kernel<G>, dim3(grid), dim3(XT_UP_WARPS * 32), p.up_smem, s, xa);
    if (dmin > 0) QW_LAUNCH_PDL("moe up (dense)", moe_up_tc_kernel, dim3(grid), dim3(TC_THREADS), TC_SMEM, s, xa);
  }
  if (down && ep) {
    if (p.down_ep_smem > GR_SMEM_LIMIT) return fail(QW_ERR_UNSUPPORTED, "moe_ep_experts: output tile does not fit");
    QW_LAUNCH_PDL("moe down (grouped, ep send)", moe_down_grouped_kernel<G, true>, dim3(grid), dim3(XT_DN_WARPS * 32),
                  p.down_ep_smem, s, xa, p.down_tps, p.down_spw, *ep);
  } else if (down) {
    QW_LAUNCH_PDL("moe down (grouped)", moe_down_grouped_kernel<G, false>, dim3(grid), dim3(XT_DN_WARPS * 32),
                  p.down_smem, s, xa, p.down_tps, p.down_spw, EpSend{});
    if (dmin > 0) QW_LAUNCH_PDL("moe down (dense)", moe_down_tc_kernel, dim3(grid), dim3(TC_THREADS), TC_SMEM, s, xa);
  }
  return QW_OK;
}

template <int G>
static int launch_experts_w4(const MoeArgs<__nv_bfloat16>& a, cudaStream_t s, bool up, bool down,
                             bool lists_ready, const EpSend* ep = nullptr) {
  const XtPlan p = xt_plan<G>(a);
  int32_t* status = nullptr;
  const int src = moe_wait_status_addr(&status);
  if (src != QW_OK) return src;
  // the bulk pair keeps h (the down input) in fp16, the streaming pair in bf16: both
  // halves of one MoE always come from the same pair
  if (!ep && p.up_ok && p.down_ok) return launch_experts_bulk<G>(a, p, s, up, down, status);
  // the grouped and streaming kernels read the lists from the workspace (built once,
  // before gate/up)
  if (up && !lists_ready) {
    const int rc = launch_route_lists(a.T, a.E, a.k, a.e_lo, a.e_cnt, a.ws, s);
    if (rc != QW_OK) return rc;
  }
  XtPlan gp{};
  if (grouped_plan<G>(a, gp)) return launch_experts_grouped<G>(a, gp, s, up, down, status, ep);
  if (ep) return fail(QW_ERR_UNSUPPORTED, "moe_ep_experts: shape outside the grouped expert kernels");
  // the arithmetic of the bulk kernels (raw-nibble gate/up, fp16 down): a token's expert
  // outputs have the same bits whichever kernels (block size) compute them
  return launch_experts<W4Fmt<G, __half>, 4, W4NibFmt<G>>(a, s, up, down);
}

}  // namespace qw

using namespace qw;

extern "C" int32_t qw_moe_dense_threshold(int32_t tokens) {
  if (tokens < 0) return g_dense_min.load();
  return g_dense_min.exchange(tokens);
}

extern "C" int64_t qw_moe_workspace_bytes(int64_t tokens, int64_t hidden, int64_t experts, int64_t inter,
                                          int64_t top_k) {
  if (tokens < 0 || hidden <= 0 || experts <= 0 || inter <= 0 || top_k <= 0) return -1;
  const int T = static_cast<int>(tokens), E = static_cast<int>(experts), k = static_cast<int>(top_k);
  int64_t b = stage_off(T, E, k) + stage_bytes(T, static_cast<int>(hidden));   // routing ints, staged x
  b += (static_cast<int64_t>(T) * k + T) * inter * 2;          // hbuf (16-bit)
  b = (b + 255) / 256 * 256;
  b += static_cast<int64_t>(T) * (k + 1) * hidden * 4;          // part
  b += static_cast<int64_t>(T) * experts * 2 + 256;             // dense-router logits
  return b;
}

struct WsParts {
  void* route;
  void* hbuf;
  float* part;
  void* logits;
};

static WsParts split_ws(void* ws, int T, int H, int E, int I, int k) {
  uint8_t* p = static_cast<uint8_t*>(ws);
  WsParts w;
  w.route = p;
  int64_t off = stage_off(T, E, k) + stage_bytes(T, H);
  w.hbuf = p + off;
  off += (static_cast<int64_t>(T) * k + T) * I * 2;
  off = (off + 255) / 256 * 256;
  w.part = reinterpret_cast<float*>(p + off);
  off += static_cast<int64_t>(T) * (k + 1) * H * 4;
  w.logits = p + off;
  return w;
}

static int route_entry(const void* logits, int logit_dtype, int64_t ldl, int64_t tokens, int64_t experts,
                       int64_t top_k, int64_t shared_col, int act_dtype, const void* x, int64_t hidden,
                       int32_t group, void* workspace, void* stream, int tie_order = 1) {
  QW_CHECK_ARG(logits && workspace, "moe_route: null pointer");
  QW_CHECK_ARG(tie_order == 0 || tie_order == 1, "moe_route: tie_order must be 0 or 1");
  QW_CHECK_ARG(tokens >= 1 && tokens <= 4096 && experts >= 1 && experts <= 1024 && top_k >= 1 &&
                   top_k <= 16 && top_k <= experts && ldl >= experts,
               "MoE needs compatible expert weights and a valid top_k");
  QW_CHECK_ARG(act_dtype == QW_BF16 || act_dtype == QW_F16, "moe_route: activation dtype");
  const int T = static_cast<int>(tokens), E = static_cast<int>(experts), k = static_cast<int>(top_k);
  int H = 0, G = 0;
  if (x != nullptr) {
    QW_CHECK_ARG(hidden >= 256 && hidden <= (1 << 20) && (group == 32 || group == 64 || group == 128),
                 "moe_route_x: invalid hidden / group");
    H = static_cast<int>(hidden);
    G = group;
    // staged only where the gate/up kernel that reads it runs (blocks of <= 16 tokens)
    // and the row layout suits a warp per token; otherwise the header says "nothing"
    if (!(T <= XT_MAXT && H % 256 == 0 && act_dtype == QW_BF16 && (reinterpret_cast<uintptr_t>(x) & 15) == 0)) x = nullptr;
  }
  if (x == nullptr) H = 256, G = 32;   // header only
  cudaStream_t s = as_stream(stream);
  const int sc = static_cast<int>(shared_col), f16 = act_dtype == QW_F16;
  if (logit_dtype == QW_BF16)
    return launch_route<__nv_bfloat16>(logits, ldl, T, E, k, sc, f16, workspace, x, H, G, s, tie_order);
  if (logit_dtype == QW_F16) return launch_route<__half>(logits, ldl, T, E, k, sc, f16, workspace, x, H, G, s, tie_order);
  if (logit_dtype == QW_F32) return launch_route<float>(logits, ldl, T, E, k, sc, f16, workspace, x, H, G, s, tie_order);
  return fail(QW_ERR_ARG, "moe_route: bad logit dtype");
}

extern "C" int qw_moe_route(const void* logits, int logit_dtype, int64_t ldl, int64_t tokens, int64_t experts,
                            int64_t top_k, int64_t shared_col, int act_dtype, void* workspace, void* stream) {
  return route_entry(logits, logit_dtype, ldl, tokens, experts, top_k, shared_col, act_dtype, nullptr, 0, 0,
                     workspace, stream);
}

extern "C" int qw_moe_route_x(const void* logits, int logit_dtype, int64_t ldl, int64_t tokens, int64_t experts,
                              int64_t top_k, int64_t shared_col, int act_dtype, const void* x, int64_t hidden,
                              int32_t group, void* workspace, void* stream, int32_t tie_order) {
  QW_CHECK_ARG(x != nullptr, "moe_route_x: null x");
  return route_entry(logits, logit_dtype, ldl, tokens, experts, top_k, shared_col, act_dtype, x, hidden, group,
                     workspace, stream, tie_order);
}

extern "C" int qw_moe_route_lists(void* workspace, int64_t tokens, int64_t experts, int64_t top_k, void* stream) {
  QW_CHECK_ARG(workspace, "moe_route_lists: null pointer");
  QW_CHECK_ARG(tokens >= 1 && tokens <= 4096 && experts >= 1 && experts <= 1024 && top_k >= 1 && top_k <= 16 &&
                   top_k <= experts, "moe_route_lists: invalid shape");
  return launch_route_lists(static_cast<int>(tokens), static_cast<int>(experts), static_cast<int>(top_k), 0,
                            static_cast<int>(experts), workspace,
                            as_stream(stream));
}

static int experts_w4(const void* x, const void* gate_up, const void* down, const void* shared_gate_up,
                      const void* shared_down, int64_t tokens, int64_t hidden, int64_t experts, int64_t inter,
                      int64_t top_k, int32_t group, void* workspace, void* stream, bool up, bool dn,
                      int64_t expert_lo = 0, int64_t expert_count = -1, bool lists_ready = false,
                      int64_t pairs_hint = 0, const EpSend* ep = nullptr) {
  if (expert_count < 0) expert_count = experts;
  QW_CHECK_ARG(x && workspace && (expert_count == 0 || (gate_up && down)), "moe_experts: null pointer");
  QW_CHECK_ARG(expert_lo >= 0 && expert_lo + expert_count <= experts, "moe_experts: expert range outside [0, experts)");
  QW_CHECK_ARG((shared_gate_up == nullptr) == (shared_down == nullptr), "moe_experts: shared expert pointers");
  QW_CHECK_ARG(group == 32 || group == 64 || group == 128, "moe_experts: group must be 32, 64 or 128");
  QW_CHECK_ARG(tokens >= 1 && tokens <= 65536 && hidden % group == 0 && inter % group == 0 && inter % 16 == 0 &&
                   hidden % 16 == 0 && top_k >= 1 && top_k <= 16 && experts >= top_k,
               "moe_experts: invalid shape");
  const int T = static_cast<int>(tokens), H = static_cast<int>(hidden), E = static_cast<int>(experts),
            I = static_cast<int>(inter), k = static_cast<int>(top_k);
  WsParts w = split_ws(workspace, T, H, E, I, k);
  MoeArgs<__nv_bfloat16> a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.gu = static_cast<const uint8_t*>(gate_up);
  a.dn = static_cast<const uint8_t*>(down);
  a.gu_stride = qw_w4_stream_bytes(2 * inter, hidden, group);
  a.dn_stride = qw_w4_stream_bytes(hidden, inter, group);
  a.sgu = static_cast<const uint8_t*>(shared_gate_up);
  a.sdn = static_cast<const uint8_t*>(shared_down);
  a.ws = w.route;
  a.hbuf = static_cast<__nv_bfloat16*>(w.hbuf);
  a.part = w.part;
  a.T = T; a.H = H; a.I = I; a.E = E; a.k = k;
  a.has_shared = shared_gate_up != nullptr;
  a.e_lo = static_cast<int>(expert_lo);
  a.e_cnt = static_cast<int>(expert_count);
  a.pairs_hint = static_cast<int>(pairs_hint);
  cudaStream_t s = as_stream(stream);
  switch (group) {
    case 128: return launch_experts_w4<128>(a, s, up, dn, lists_ready, ep);
    case 64: return launch_experts_w4<64>(a, s, up, dn, lists_ready, ep);
    default: return launch_experts_w4<32>(a, s, up, dn, lists_ready, ep);
  }
}

extern "C" int qw_moe_experts_w4(const void* x, const void* gate_up, const void* down,
                                 const void* shared_gate_up, const void* shared_down, int64_t tokens,
                                 int64_t hidden, int64_t experts, int64_t inter, int64_t top_k,
                                 int32_t group, void* workspace, void* stream) {
  return experts_w4(x, gate_up, down, shared_gate_up, shared_down, tokens, hidden, experts, inter, top_k, group,
                    workspace, stream, true, true);
}

extern "C" int qw_moe_experts_w4_range(const void* x, const void* gate_up, const void* down,
                                       const void* shared_gate_up, const void* shared_down, int64_t tokens,
                                       int64_t hidden, int64_t experts, int64_t inter, int64_t top_k, int32_t group,
                                       int64_t expert_lo, int64_t expert_count, void* workspace, void* stream) {
  return experts_w4(x, gate_up, down, shared_gate_up, shared_down, tokens, hidden, experts, inter, top_k, group,
                    workspace, stream, true, true, expert_lo, expert_count);
}

extern "C" int qw_moe_up_w4(const void* x, const void* gate_up, const void* down, const void* shared_gate_up,
                            const void* shared_down, int64_t tokens, int64_t hidden, int64_t experts,
                            int64_t inter, int64_t top_k, int32_t group, void* workspace, void* stream) {
  return experts_w4(x, gate_up, down, shared_gate_up, shared_down, tokens, hidden, experts, inter, top_k, group,
                    workspace, stream, true, false);
}

extern "C" int qw_moe_down_w4(const void* x, const void* gate_up, const void* down, const void* shared_gate_up,
                              const void* shared_down, int64_t tokens, int64_t hidden, int64_t experts,
                              int64_t inter, int64_t top_k, int32_t group, void* workspace, void* stream) {
  return experts_w4(x, gate_up, down, shared_gate_up, shared_down, tokens, hidden, experts, inter, top_k, group,
                    workspace, stream, false, true);
}

extern "C" int32_t qw_moe_active_experts(const void* workspace, int64_t tokens, int64_t experts, int64_t top_k) {
  // host helper for measurement: byte offset of the active-expert count in the workspace
  (void)workspace;
  const int T = static_cast<int>(tokens), E = static_cast<int>(experts), k = static_cast<int>(top_k);
  return static_cast<int32_t>((2LL * T * k + T) * 4 + 0 * E);
}

extern "C" int qw_moe_partials(void* workspace, int64_t tokens, int64_t hidden, int64_t experts,
                               int64_t inter, int64_t top_k, const float** part, const int32_t** topk_idx,
                               const float** topk_w, const float** shared_gate) {
  QW_CHECK_ARG(workspace, "moe_partials: null workspace");
  const int T = static_cast<int>(tokens), E = static_cast<int>(experts), k = static_cast<int>(top_k);
  WsParts w = split_ws(workspace, T, static_cast<int>(hidden), E, static_cast<int>(inter), k);
  RouteView rv = route_view(w.route, T, E, k);
  if (part) *part = w.part;
  if (topk_idx) *topk_idx = rv.topk_idx;
  if (topk_w) *topk_w = rv.topk_w;
  if (shared_gate) *shared_gate = rv.shared_gate;
  return QW_OK;
}

extern "C" int qw_moe_combine(void* workspace, void* out, int residual, int64_t tokens, int64_t hidden,
                              int64_t experts, int64_t inter, int64_t top_k, int has_shared, void* stream) {
  QW_CHECK_ARG(workspace && out, "moe_combine: null pointer");
  QW_CHECK_ARG(tokens >= 1 && top_k >= 1 && top_k <= 32 && hidden > 0, "moe_combine: invalid shape");
  const int T = static_cast<int>(tokens), H = static_cast<int>(hidden), E = static_cast<int>(experts),
            I = static_cast<int>(inter), k = static_cast<int>(top_k);
  WsParts w = split_ws(workspace, T, H, E, I, k);
  moe_combine_kernel<__nv_bfloat16><<<T, 256, 0, as_stream(stream)>>>(
      w.part, w.route, static_cast<__nv_bfloat16*>(out), T, H, E, k, has_shared, residual);
  QW_LAUNCH_CHECK("moe combine");
  return QW_OK;
}

static int combine_norm_entry(void* workspace, void* hidden, int64_t tokens, int64_t hidden_dim, int64_t experts,
                              int64_t inter, int64_t top_k, int has_shared, const void* gamma, void* normed, float eps,
                              void* tap, int64_t ldf, int tap_normed, void* stream, EpRecv ep_recv) {
  QW_CHECK_ARG(workspace && hidden && gamma && normed, "moe_combine_norm: null pointer");
  QW_CHECK_ARG(tokens >= 1 && top_k >= 1 && top_k <= 16 && hidden_dim > 0 && hidden_dim % 4 == 0 && eps > 0.f,
               "moe_combine_norm: invalid shape");
  QW_CHECK_ARG(!tap || (ldf >= hidden_dim && ldf % 4 == 0 && (reinterpret_cast<uintptr_t>(tap) & 7) == 0),
               "moe_combine_norm: tap rows must be 8-byte aligned (ldf a multiple of 4)");
  QW_CHECK_ARG(((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(normed) |
                 reinterpret_cast<uintptr_t>(gamma)) & 7) == 0,
               "moe_combine_norm: hidden, normed and gamma must be 8-byte aligned");
  const int T = static_cast<int>(tokens), H = static_cast<int>(hidden_dim), E = static_cast<int>(experts),
            I = static_cast<int>(inter), k = static_cast<int>(top_k);
  WsParts w = split_ws(workspace, T, H, E, I, k);
  QW_CHECK_ARG((reinterpret_cast<uintptr_t>(w.part) & 15) == 0, "moe_combine_norm: workspace alignment");
  cudaStream_t s = as_stream(stream);
  auto* hp = static_cast<__nv_bfloat16*>(hidden);
  auto* gp = static_cast<const __nv_bfloat16*>(gamma);
  auto* np_ = static_cast<__nv_bfloat16*>(normed);
  auto* tp = static_cast<__nv_bfloat16*>(tap);
  const float* part = w.part;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(T * CN_SPLIT);
  cfg.blockDim = dim3(CN_THREADS);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CN_SPLIT;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = k <= 8 ? cudaLaunchKernelEx(&cfg, moe_combine_norm_kernel<8>, part, w.route, hp, T, H, E, k,
                                                    has_shared, gp, np_, eps, tp, ldf, tap_normed, ep_recv)
                               : cudaLaunchKernelEx(&cfg, moe_combine_norm_kernel<16>, part, w.route, hp, T, H, E, k,
                                                    has_shared, gp, np_, eps, tp, ldf, tap_normed, ep_recv);
  if (e != cudaSuccess) return cuda_status(e, "moe combine_norm");
  return QW_OK;
}

extern "C" int qw_moe_combine_norm(void* workspace, void* hidden, int64_t tokens, int64_t hidden_dim,
                                   int64_t experts, int64_t inter, int64_t top_k, int has_shared,
                                   const void* gamma, void* normed, float eps, void* tap, int64_t ldf,
                                   int tap_normed, void* stream) {
  return combine_norm_entry(workspace, hidden, tokens, hidden_dim, experts, inter, top_k, has_shared, gamma, normed,
                            eps, tap, ldf, tap_normed, stream, EpRecv{});
}

extern "C" int qw_moe_ep_combine_norm(void* workspace, void* window, int64_t ranks, int64_t cap, void* hidden,
                                      int64_t tokens, int64_t hidden_dim, int64_t experts, int64_t inter,
                                      int64_t top_k, int has_shared, const void* gamma, void* normed, float eps,
                                      void* tap, int64_t ldf, int tap_normed, void* stream) {
  QW_CHECK_ARG(window, "moe_ep_combine_norm: null window");
  QW_CHECK_ARG(ranks >= 1 && ranks <= EP_MAX_RANKS && cap == tokens * (top_k + (has_shared ? 1 : 0)) &&
                   hidden_dim % 8 == 0, "moe_ep_combine_norm: shape (cap = tokens * (top_k + shared))");
  return combine_norm_entry(workspace, hidden, tokens, hidden_dim, experts, inter, top_k, has_shared, gamma, normed,
                            eps, tap, ldf, tap_normed, stream,
                            EpRecv{window, static_cast<int>(ranks), static_cast<int>(cap)});
}

extern "C" int qw_moe(const void* hidden, const void* router, const void* gate_up, const void* down, void* out,
                      int dtype, int64_t tokens, int64_t hidden_dim, int64_t experts, int64_t inter,
                      int64_t top_k, int32_t* topk_idx_out, void* workspace, void* stream) {
  QW_CHECK_ARG(hidden && router && gate_up && down && out && workspace, "moe: null pointer");
  QW_CHECK_ARG(dtype == QW_BF16 || dtype == QW_F16, "moe: bf16 or fp16 tensors required");
  QW_CHECK_ARG(tokens >= 1 && tokens <= 4096 && experts >= 1 && experts <= 1024 && top_k >= 1 && top_k <= 16 &&
                   top_k <= experts && hidden_dim % 16 == 0 && inter % 16 == 0 && hidden_dim > 0 && inter > 0,
               "MoE needs compatible expert weights and a valid top_k");
  const int T = static_cast<int>(tokens), H = static_cast<int>(hidden_dim), E = static_cast<int>(experts),
            I = static_cast<int>(inter), k = static_cast<int>(top_k);
  cudaStream_t s = as_stream(stream);
  WsParts w = split_ws(workspace, T, H, E, I, k);
  const int warps = T * E;
  const unsigned rblocks = static_cast<unsigned>((warps * 32 + 255) / 256);
  int st;
  if (dtype == QW_BF16) {
    router_dense_kernel<__nv_bfloat16><<<rblocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(hidden), static_cast<const __nv_bfloat16*>(router),
        static_cast<__nv_bfloat16*>(w.logits), T, H, E);
    QW_LAUNCH_CHECK("moe router");
    st = launch_route<__nv_bfloat16>(w.logits, E, T, E, k, -1, 0, w.route, nullptr, 256, 32, s);
  } else {
    router_dense_kernel<__half><<<rblocks, 256, 0, s>>>(static_cast<const __half*>(hidden),
                                                        static_cast<const __half*>(router),
                                                        static_cast<__half*>(w.logits), T, H, E);
    QW_LAUNCH_CHECK("moe router");
    st = launch_route<__half>(w.logits, E, T, E, k, -1, 1, w.route, nullptr, 256, 32, s);
  }
  if (st) return st;
  st = launch_route_lists(T, E, k, 0, E, w.route, s);
  if (st) return st;
  if (dtype == QW_BF16) {
    MoeArgs<__nv_bfloat16> a{};
    a.x = static_cast<const __nv_bfloat16*>(hidden);
    a.gu = static_cast<const uint8_t*>(gate_up);
    a.dn = static_cast<const uint8_t*>(down);
    a.gu_stride = 2LL * I * H * 2; a.dn_stride = 1LL * H * I * 2;
    a.gu_ld = 2LL * H; a.dn_ld = 2LL * I;
    a.ws = w.route; a.hbuf = static_cast<__nv_bfloat16*>(w.hbuf); a.part = w.part;
    a.T = T; a.H = H; a.I = I; a.E = E; a.k = k; a.has_shared = 0; a.e_lo = 0; a.e_cnt = E;
    st = launch_experts<RowFmt<__nv_bfloat16>, 2>(a, s, true, true);
    if (st) return st;
    moe_combine_kernel<__nv_bfloat16><<<T, 256, 0, s>>>(w.part, w.route, static_cast<__nv_bfloat16*>(out), T, H, E, k, 0, 0);
  } else {
    MoeArgs<__half> a{};
    a.x = static_cast<const __half*>(hidden);
    a.gu = static_cast<const uint8_t*>(gate_up);
    a.dn = static_cast<const uint8_t*>(down);
    a.gu_stride = 2LL * I * H * 2; a.dn_stride = 1LL * H * I * 2;
    a.gu_ld = 2LL * H; a.dn_ld = 2LL * I;
    a.ws = w.route; a.hbuf = static_cast<__half*>(w.hbuf); a.part = w.part;
    a.T = T; a.H = H; a.I = I; a.E = E; a.k = k; a.has_shared = 0; a.e_lo = 0; a.e_cnt = E;
    st = launch_experts<RowFmt<__half>, 2>(a, s, true, true);
    if (st) return st;
    moe_combine_kernel<__half><<<T, 256, 0, s>>>(w.part, w.route, static_cast<__half*>(out), T, H, E, k, 0, 0);
  }
  QW_LAUNCH_CHECK("moe combine");
  if (topk_idx_out) {
    RouteView rv = route_view(w.route, T, E, k);
    cudaError_t e = cudaMemcpyAsync(topk_idx_out, rv.topk_idx, sizeof(int32_t) * T * k, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return cuda_status(e, "moe topk copy");
  }
  return QW_OK;
}

// ------------------------------------------------------------------ expert parallelism
// Experts sharded over G ranks (rank g owns experts [g E/G, (g+1) E/G)): each rank routes
// its own tokens over all E experts, sends every (token, slot) pair's activation row to
// the owning rank, each rank runs its local experts on the rows it received, and the
// results come back to the source rank's per-(token, slot) outputs, where the usual
// combine reads them.
//
// The exchange is device-initiated over NVLink: every rank holds one window (a device
// allocation that every peer has mapped, qw_ep_window_*), and the kernels store straight
// into the peers' windows -- rows and their descriptors on dispatch, results on
// combine -- then raise a flag in each peer's window with a system-scope release; the
// consumer's kernel waits (bounded) on the flags in its own window with acquire loads.
// Only the routed rows travel (no fixed-size segments), there is no host round trip
// and no collective library on the data path, and the kernels are stream-ordered, so a
// whole verify step with its exchanges replays as one CUDA graph.  No TMA and no
// multicast touches peer memory: plain 16-byte stores from SM threads.
//
// Window of rank g (identical layout on every rank):
//   hdr   int32[64]   [0] epoch of the last closed exchange, [3] CTA ticket of the
//                     kernel that closes it, [4] broken (a wait expired)
//   dcnt  u64[64]     rows arrived from source s (+ its count message), EP_ROUND each
//                     exchange
//   ccnt  u64[64]     result pieces arrived from expert owner d (+ its count message)
//   count int32[64]   count[s] = rows source s sent to g in the current exchange
//   meta  int32[G][cap]       (source pair index << 9) | local expert, per received row
//   rows  bf16 [G][cap][H]    received rows (source s at rows [s][0, count[s]))
//   back  bf16 [cap][H]       this rank's own pairs' expert outputs (pair p at row p)
// With the shared expert exchanged too (shared = 1), every rank holds it as local expert
// el = E/G after its routed ones, and each token sends one more pair (index T k + t) to
// its own rank: the shared expert then runs in the same launches as the routed ones.
// Ordering: a rank's scatter of exchange n waits for every peer's combine of n, so its
// dispatch of n + 1 cannot overwrite a window region a peer is still reading.
//
// Every expert output is computed by the same kernels as on one GPU (they give a row the
// same bits whatever else is in the launch) and crosses ranks as bf16, the precision
// the combine reads it at, so the result is bit-identical to the single-GPU MoE.
namespace qw {

// Position of pair p in its destination's rows: the earlier pairs with the same
// destination, counted by the whole CTA (every thread calls it with the same p).
__device__ __forceinline__ int ep_pos(const int32_t* idx, int p, int d, int el) {
  int pos = 0;
  for (int q0 = 0; q0 < p; q0 += blockDim.x) {
    const int q = q0 + threadIdx.x;
    pos += __syncthreads_count(q < p && idx[q] / el == d);
  }
  return pos;
}

// Destination of routed pair p and its position among the pairs to that destination,
// counted by the whole CTA.  Shared-expert pairs (p >= T k: token p - T k) stay on this
// rank, after its routed pairs.
__device__ __forceinline__ void ep_route_pair(const int32_t* idx, int p, int np, int el, int rank, int& d, int& pos) {
  if (p < np) {
    d = idx[p] / el;
    pos = ep_pos(idx, p, d, el);
  } else {
    d = rank;
    int before = 0;
    for (int q0 = 0; q0 < np; q0 += blockDim.x) {
      const int q = q0 + threadIdx.x;
      before += __syncthreads_count(q < np && idx[q] / el == rank);
    }
    pos = before + (p - np);
  }
}

// Dispatch (source rank): one CTA per pair -- the T k routed pairs, then (with the shared
// expert, local expert el of every rank) one per token -- stores its token's row and
// descriptor into the owner's window; the last CTA stores the per-destination counts and
// raises this rank's dispatch flag in every window (all ranks, rows or not).
__global__ void ep_dispatch_kernel(const int32_t* __restrict__ idx, const __nv_bfloat16* __restrict__ x, int T, int H,
                                   int k, int G, int rank, int el, int shared, int cap,
                                   const unsigned long long* __restrict__ peers, void* own) {
  pdl_wait();
  pdl_trigger();
  const EpWin me = ep_win(own, G, cap, H);
  const int epoch = me.hdr[0] + 1;
  const int np = T * k;
  const int p = blockIdx.x;
  int d, pos;
  ep_route_pair(idx, p, np, el, rank, d, pos);
  const int tok = p < np ? p / k : p - np;
  const int local = p < np ? idx[p] - d * el : el;
  const EpWin dst = ep_win(reinterpret_cast<const void*>(peers[d]), G, cap, H);
  if (threadIdx.x == 0) dst.meta[rank * cap + pos] = (p << 9) | local;
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(tok) * H);
  uint4* out = reinterpret_cast<uint4*>(dst.rows + (static_cast<int64_t>(rank) * cap + pos) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) out[i] = src[i];
  __syncthreads();
  if (threadIdx.x == 0) red_release_sys(dst.dcnt + rank, 1ull);   // after the row and its descriptor
  if (blockIdx.x != 0) return;
  // CTA 0: the counts, then each destination's complement to EP_ROUND
  for (int g = 0; g < G; ++g) {
    int c = 0;
    for (int q0 = 0; q0 < np; q0 += blockDim.x) {
      const int q = q0 + threadIdx.x;
      c += __syncthreads_count(q < np && idx[q] / el == g);
    }
    if (threadIdx.x == 0) {
      c += (g == rank && shared) ? T : 0;
      const EpWin w = ep_win(reinterpret_cast<const void*>(peers[g]), G, cap, H);
      w.count[rank] = c;
      red_release_sys(w.dcnt + rank, EP_ROUND - static_cast<unsigned long long>(c));
    }
  }
  (void)epoch;
}

// Receiving rank: wait for every source's dispatch, then route the received rows
// (top-1 = the row's local expert, weight 1) and build the expert lists over the valid
// rows only (compacted), with each list entry naming the row's place in the window.
// One CTA; dynamic smem: 3 el + 64 ints.
__global__ void __launch_bounds__(1024) ep_recv_route_kernel(void* own, int G, int cap, int H, int el, void* ws) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ int s_cnt[EP_MAX_RANKS], s_off[EP_MAX_RANKS + 1];
  pdl_wait();
  pdl_trigger();
  const EpWin me = ep_win(own, G, cap, H);
  const int epoch = me.hdr[0] + 1;
  if (threadIdx.x < G) {
    const bool ok = ep_wait_count(me.dcnt + threadIdx.x, static_cast<unsigned long long>(epoch) * EP_ROUND, me.hdr);
    const int c = ok ? __ldcg(me.count + threadIdx.x) : 0;
    s_cnt[threadIdx.x] = c < 0 ? 0 : (c > cap ? cap : c);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    s_off[0] = 0;
    for (int g = 0; g < G; ++g) s_off[g + 1] = s_off[g] + s_cnt[g];
  }
  __syncthreads();
  const int n = s_off[G];
  const RouteView rv = route_view(ws, G * cap, el, 1);
  int* phys = reinterpret_cast<int*>(rv.topk_w);   // [n] window row of each compacted row
  for (int c = threadIdx.x; c < n; c += blockDim.x) {
    int src = 0;
    while (c >= s_off[src + 1]) ++src;
    const int j = c - s_off[src];
    const int le = __ldcg(me.meta + src * cap + j) & 0x1FF;
    rv.topk_idx[c] = le < el ? le : -1;
    phys[c] = src * cap + j;
  }
  __syncthreads();
  int* scratch = reinterpret_cast<int*>(smem);
  build_route_lists(rv.topk_idx, n, el, 1, 0, scratch, scratch + 3 * el, rv.n_active, rv.active, rv.pair_off,
                    rv.pair_tok, rv.pair_slot);
  __syncthreads();
  const int listed = rv.pair_off[*rv.n_active];
  for (int i = threadIdx.x; i < listed; i += blockDim.x) rv.pair_tok[i] = phys[rv.pair_tok[i]];
}

// Scatter (source rank): wait for every rank's combine, then the returned rows into the
// source routing's per-(token, slot) outputs (a shared-expert pair p >= T k into slot k
// of token p - T k); the last CTA closes the exchange (epoch).
__global__ void ep_scatter_kernel(void* own, int T, int H, int k, int G, int cap, float* __restrict__ part) {
  __shared__ int s_ok;
  pdl_wait();
  pdl_trigger();
  const EpWin me = ep_win(own, G, cap, H);
  const int epoch = me.hdr[0] + 1;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < G && !ep_wait_count(me.ccnt + threadIdx.x, static_cast<unsigned long long>(epoch) * EP_ROUND,
                                        me.hdr))
    s_ok = 0;
  __syncthreads();
  const int p = blockIdx.x;
  if (s_ok) {
    const __nv_bfloat16* src = me.back + static_cast<int64_t>(p) * H;
    const int np = T * k;
    const int64_t slot_row = p < np ? static_cast<int64_t>(p / k) * (k + 1) + p % k
                                    : static_cast<int64_t>(p - np) * (k + 1) + k;
    float* dst = part + slot_row * H;
    for (int i = threadIdx.x; i < H / 2; i += blockDim.x) {
      const unsigned u = __ldcg(reinterpret_cast<const unsigned*>(src) + i);
      const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
      *reinterpret_cast<float2*>(dst + 2 * i) = v;
    }
  }
  if (ep_last_cta(me.hdr + 3) && threadIdx.x == 0) me.hdr[0] = epoch;
}

static int ep_check(int64_t tokens, int64_t hidden, int64_t experts, int64_t top_k, int64_t ranks, int64_t cap,
                    int shared) {
  QW_CHECK_ARG(tokens >= 1 && tokens * top_k <= 4096 && top_k >= 1 && top_k <= 16 && hidden % 8 == 0 && hidden > 0,
               "moe_ep: invalid shape (tokens * top_k <= 4096, hidden % 8 == 0)");
  QW_CHECK_ARG(ranks >= 1 && ranks <= EP_MAX_RANKS && experts % ranks == 0 && experts / ranks <= 256,
               "moe_ep: 1 <= ranks <= 64, experts must split evenly, <= 256 per rank");
  QW_CHECK_ARG(shared == 0 || shared == 1, "moe_ep: shared must be 0 or 1");
  QW_CHECK_ARG(cap == tokens * (top_k + shared),
               "moe_ep: cap must be tokens * (top_k + shared) (the rows one source can send)");
  return QW_OK;
}

}  // namespace qw

extern "C" int64_t qw_ep_window_bytes(int64_t ranks, int64_t cap, int64_t hidden) {
  if (ranks <= 0 || ranks > EP_MAX_RANKS || cap <= 0 || hidden <= 0) return -1;
  return ep_window_bytes(static_cast<int>(ranks), static_cast<int>(cap), static_cast<int>(hidden));
}

extern "C" int qw_ep_window_alloc(int64_t bytes, void** window, void* ipc_handle) {
  QW_CHECK_ARG(bytes > 0 && window && ipc_handle, "ep_window_alloc: invalid argument");
  void* p = nullptr;
  cudaError_t err = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (err != cudaSuccess) return cuda_status(err, "ep_window_alloc: cudaMalloc");
  err = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (err == cudaSuccess) err = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (err != cudaSuccess) {
    cudaFree(p);
    return cuda_status(err, "ep_window_alloc: clear / IPC handle");
  }
  *window = p;
  return QW_OK;
}

extern "C" int qw_ep_window_open(const void* ipc_handle, void** peer_window) {
  QW_CHECK_ARG(ipc_handle && peer_window, "ep_window_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t err = cudaIpcOpenMemHandle(peer_window, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return cuda_status(err, "ep_window_open: cudaIpcOpenMemHandle");
  return QW_OK;
}

extern "C" int qw_ep_window_close(void* peer_window) {
  QW_CHECK_ARG(peer_window, "ep_window_close: null pointer");
  const cudaError_t err = cudaIpcCloseMemHandle(peer_window);
  if (err != cudaSuccess) return cuda_status(err, "ep_window_close");
  return QW_OK;
}

extern "C" int qw_ep_window_free(void* window) {
  QW_CHECK_ARG(window, "ep_window_free: null pointer");
  const cudaError_t err = cudaFree(window);
  if (err != cudaSuccess) return cuda_status(err, "ep_window_free");
  return QW_OK;
}

extern "C" int64_t qw_moe_ep_recv_workspace_bytes(int64_t ranks, int64_t cap, int64_t hidden, int64_t local_experts,
                                                  int64_t inter) {
  if (ranks <= 0 || cap <= 0 || local_experts <= 0) return -1;
  return qw_moe_workspace_bytes(ranks * cap, hidden, local_experts, inter, 1);
}

extern "C" int qw_moe_ep_dispatch(const void* workspace, const void* x, int64_t tokens, int64_t hidden,
                                  int64_t experts, int64_t top_k, int64_t ranks, int64_t rank, int64_t cap,
                                  int shared, const void* peers, void* window, void* stream) {
  QW_CHECK_ARG(workspace && x && peers && window, "moe_ep_dispatch: null pointer");
  const int st = ep_check(tokens, hidden, experts, top_k, ranks, cap, shared);
  if (st) return st;
  QW_CHECK_ARG(rank >= 0 && rank < ranks, "moe_ep_dispatch: rank outside [0, ranks)");
  QW_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0, "moe_ep_dispatch: x must be 16-byte aligned");
  const int T = static_cast<int>(tokens), E = static_cast<int>(experts), k = static_cast<int>(top_k);
  const RouteView rv = route_view(const_cast<void*>(workspace), T, E, k);
  QW_LAUNCH_PDL("moe ep dispatch", ep_dispatch_kernel, dim3(static_cast<unsigned>(cap)), dim3(256), 0,
                as_stream(stream), rv.topk_idx, static_cast<const __nv_bfloat16*>(x), T, static_cast<int>(hidden), k,
                static_cast<int>(ranks), static_cast<int>(rank), static_cast<int>(experts / ranks), shared,
                static_cast<int>(cap), static_cast<const unsigned long long*>(peers), window);
  return QW_OK;
}

extern "C" int qw_moe_ep_recv_route(void* window, int64_t ranks, int64_t cap, int64_t hidden, int64_t local_experts,
                                    void* recv_workspace, void* stream) {
  QW_CHECK_ARG(window && recv_workspace, "moe_ep_recv_route: null pointer");
  QW_CHECK_ARG(ranks >= 1 && ranks <= EP_MAX_RANKS && cap >= 1 && local_experts >= 1 && local_experts <= 257,
               "moe_ep_recv_route: shape");
  const int el = static_cast<int>(local_experts);
  const size_t smem = (3 * static_cast<size_t>(el) + 64) * sizeof(int);
  QW_LAUNCH_PDL("moe ep recv route", ep_recv_route_kernel, dim3(1), dim3(1024), smem, as_stream(stream), window,
                static_cast<int>(ranks), static_cast<int>(cap), static_cast<int>(hidden), el, recv_workspace);
  return QW_OK;
}

extern "C" int qw_moe_ep_experts(void* window, const void* gate_up_local, const void* down_local, int64_t ranks,
                                 int64_t rank, int64_t cap, int64_t hidden, int64_t local_experts, int64_t inter,
                                 int32_t group, const void* peers, void* recv_workspace, void* stream) {
  QW_CHECK_ARG(window && peers && recv_workspace, "moe_ep_experts: null pointer");
  QW_CHECK_ARG(ranks >= 1 && ranks <= EP_MAX_RANKS && rank >= 0 && rank < ranks && cap >= 1 && local_experts >= 1 &&
                   local_experts <= 257, "moe_ep_experts: shape");
  // the window's received rows as ranks * cap rows, routed (lists included) by
  // qw_moe_ep_recv_route; the down projection sends its outputs to their sources
  const EpWin w = ep_win(window, static_cast<int>(ranks), static_cast<int>(cap), static_cast<int>(hidden));
  const EpSend ep{window, static_cast<const unsigned long long*>(peers), static_cast<int>(ranks),
                  static_cast<int>(rank), static_cast<int>(cap)};
  return experts_w4(w.rows, gate_up_local, down_local, nullptr, nullptr, ranks * cap, hidden, local_experts, inter,
                    1, group, recv_workspace, stream, true, true, 0, local_experts, true, cap, &ep);
}

extern "C" int qw_moe_ep_scatter(void* workspace, void* window, int64_t tokens, int64_t hidden, int64_t experts,
                                 int64_t inter, int64_t top_k, int64_t ranks, int64_t cap, int shared, void* stream) {
  QW_CHECK_ARG(workspace && window, "moe_ep_scatter: null pointer");
  const int st = ep_check(tokens, hidden, experts, top_k, ranks, cap, shared);
  if (st) return st;
  const int T = static_cast<int>(tokens), H = static_cast<int>(hidden), E = static_cast<int>(experts),
            k = static_cast<int>(top_k);
  WsParts w = split_ws(workspace, T, H, E, static_cast<int>(inter), k);
  QW_LAUNCH_PDL("moe ep scatter", ep_scatter_kernel, dim3(static_cast<unsigned>(cap)), dim3(256), 0,
                as_stream(stream), window, T, H, k, static_cast<int>(ranks), static_cast<int>(cap), w.part);
  return QW_OK;
}
