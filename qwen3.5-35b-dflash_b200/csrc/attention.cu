// Causal GQA attention of the verify block against the KV cache
// (reference/fused_ops.py:127-145; fused/model.py:278-294).
//
// split kernel   CTA = (key split, kv head x row group, sequence).  The G query heads
//                sharing a KV head and the S block positions form up to 128 query rows
//                (16 per warp); K/V tiles of 32 keys are staged in shared memory and both
//                products run on mma.sync (Q K^T with K as the col-major B operand,
//                P V with V through ldmatrix.trans).  Online softmax in fp32; P is
//                rounded to the activation dtype for the PV product.  Each split writes
//                its unnormalized output, row max and row sum.
// combine kernel merges the splits, rounds to the activation dtype and, for the model's
//                gated attention (fused/model.py:293), multiplies by sigmoid(gate).
// prep kernel    q/k RMSNorm with zero-centred weights (:282-283), partial RoPE
//                (:265-276, fp32 angles rounded to the activation dtype), and the append
//                of the block's K/V into the paged cache (the CacheUpdate role, :286).
//
// KV addressing: element (page, kv head, slot in page, d) of a cache at
// base + ((page * Hkv + kvh) * P + slot) * D + d.  A sequence's position t lives in page
// pages[b * max_pages + t / P].  The fused-ops operator's ND cache [B, Hkv, T, D] is the
// case P = T with page b.
#include <mutex>

#include "qw_common.cuh"

namespace qw {

constexpr int ATT_KT = 32;       // keys per tile
constexpr int ATT_MAXROWS = 64;  // query rows per CTA
constexpr int ATT_NST = 3;        // K/V tile stages in flight
constexpr int ATT_MIN_KC = 128;   // keys per split at least (partials cost about as much as the keys)
constexpr int ATT_PGCAP = 64;     // page indices staged per CTA

template <typename ET>
struct AttnArgs {
  const ET* q;
  int64_t qb, qh, qs;          // query strides (elements) for (b, h, s); d contiguous
  const ET* k;
  const ET* v;
  const int32_t* pages;        // [B, max_pages] or null (page = b)
  int max_pages, P;
  const int32_t* qpos;         // [B] first query position, or null -> qpos_scalar
  int qpos_scalar;
  int B, H, Hkv, S, kc, nsplit, rowgroups;
  float scale;
  float* opart;                // [nsplit, B, H, S, D]
  float* ml;                   // [nsplit, B, H, S, 2]
  int pgcap;                   // page indices a CTA may stage in shared memory
  int block_full;              // 1: every query row sees the whole block (no causal order inside it)
  int window;                  // > 0: row at position p sees keys > p - window only
  int plog2;                   // log2(P) when P is a power of two, else -1
};

__device__ __forceinline__ uint32_t pack2(float lo, float hi, bool f16) {
  if (f16) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

template <typename ET, int D>
__global__ void __launch_bounds__(256) attn_split_kernel(AttnArgs<ET> a) {
  constexpr int XS = D + 8;  // smem row stride (elements)
  extern __shared__ __align__(16) uint8_t smem[];
  ET* qsm = reinterpret_cast<ET*>(smem);                 // [128][XS]
  ET* ksm = qsm + ATT_MAXROWS * XS;                      // ATT_NST stages of K [32][XS], V [32][XS]
  int* pg = reinterpret_cast<int*>(ksm + ATT_NST * 2 * ATT_KT * XS);  // [pgcap] page of each key page
  // q and the block's own keys come from the predecessor (prep); the page table, the
  // query positions and the keys of earlier steps are older, so the first K/V tiles of
  // the context are requested before the wait
  const int split = blockIdx.x;
  const int kvh = blockIdx.y / a.rowgroups, rg = blockIdx.y % a.rowgroups;
  const int b = blockIdx.z;
  const int G = a.H / a.Hkv;
  const int R = G * a.S;
  const int row0 = rg * ATT_MAXROWS;
  const int nrows = min(ATT_MAXROWS, R - row0);
  const int qpos = a.qpos ? a.qpos[b] : a.qpos_scalar;
  const int len = qpos + a.S;
  const int k0 = split * a.kc;
  if (k0 >= len) return;
  const int k1 = min(len, k0 + a.kc);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const bool f16 = std::is_same<ET, __half>::value;

  // page of every key page this CTA reads (staged when it fits)
  const int p0 = k0 / a.P, npg = (k1 - 1) / a.P - p0 + 1;
  const bool staged = npg <= a.pgcap;
  if (staged)
    for (int i = threadIdx.x; i < npg; i += blockDim.x) pg[i] = a.pages ? a.pages[b * a.max_pages + p0 + i] : b;
  __syncthreads();
  // Rows are copied by warps, a row's 16-byte chunks by lanes: a lane's row offset is
  // computed once per row, with a shift and a mask for a power-of-two page size (the
  // row loops are unrolled, so the page-table reads of a warp's rows overlap).
  constexpr int CPR = D / 8;      // 16-byte chunks of one row
  constexpr int RPI = 32 / CPR;   // rows one warp instruction covers
  const int rsub = lane / CPR, cc = (lane % CPR) * 8;
  auto key_off = [&](int t) -> int64_t {
    const int pi = a.plog2 >= 0 ? (t >> a.plog2) : t / a.P;
    const int ps = t - pi * a.P;
    const int page = staged ? pg[pi - p0] : (a.pages ? a.pages[b * a.max_pages + pi] : b);
    return ((static_cast<int64_t>(page) * a.Hkv + kvh) * a.P + ps) * D;
  };
  // K/V tile t0.. -> stage st (keys past k1 zero-filled)
  auto load_tile = [&](int st, int t0) {
    ET* kd = ksm + st * 2 * ATT_KT * XS;
    ET* vd = kd + ATT_KT * XS;
#pragma unroll 8
    for (int r = warp * RPI + rsub; r < ATT_KT; r += nwarps * RPI) {
      const bool valid = t0 + r < k1;
      const int64_t off = key_off(valid ? t0 + r : k0) + cc;
      cp_async16(kd + r * XS + cc, a.k + off, valid);
      cp_async16(vd + r * XS + cc, a.v + off, valid);
    }
  };
  const int ntiles = (k1 - k0 + ATT_KT - 1) / ATT_KT;
  // the first ATT_NST - 1 tiles, one cp.async group each: those wholly before qpos now
  int pre = 0;
  while (pre < ATT_NST - 1 && pre < ntiles && k0 + (pre + 1) * ATT_KT <= qpos) {
    load_tile(pre, k0 + pre * ATT_KT);
    cp_async_commit();
    ++pre;
  }
  pdl_wait();
  pdl_trigger();
  for (int st = pre; st < ATT_NST - 1; ++st) {
    if (st < ntiles) load_tile(st, k0 + st * ATT_KT);
    cp_async_commit();
  }
  // Q rows -> smem (row r: head kvh*G + (row0+r)/S, position (row0+r)%S)
#pragma unroll 4
  for (int r = warp * RPI + rsub; r < nwarps * 16; r += nwarps * RPI) {
    const bool valid = r < nrows;
    const int rr = row0 + (valid ? r : 0);
    const int h = kvh * G + rr / a.S, s = rr % a.S;
    cp_async16(qsm + r * XS + cc, a.q + b * a.qb + h * a.qh + s * a.qs + cc, valid);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();

  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int wrow = warp * 16;
  int smax[2], smin[2];  // last and first visible key for the lane's two rows
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2) {
    const int rr = row0 + wrow + gid + 8 * h2;
    const int qp = qpos + rr % a.S;
    smax[h2] = (wrow + gid + 8 * h2 < nrows) ? (a.block_full ? qpos + a.S - 1 : qp) : -1;
    smin[h2] = a.window > 0 ? qp - a.window + 1 : 0;
  }
  // ldmatrix row addresses
  const int qa_row = wrow + ((lane >> 3) & 1) * 8 + (lane & 7);
  const int qa_col = (lane >> 4) * 8;
  const int kb_key = (lane >> 4) * 8 + (lane & 7);
  const int kb_col = ((lane >> 3) & 1) * 8;
  const int vb_key = ((lane >> 3) & 1) * 8 + (lane & 7);
  const int vb_col = (lane >> 4) * 8;

  for (int it = 0; it < ntiles; ++it) {
    const int t0 = k0 + it * ATT_KT;
    cp_async_wait<ATT_NST - 2>();
    __syncthreads();  // tile it landed for every thread; stage (it - 1) % NST is free
    {
      const int nt = it + ATT_NST - 1;
      if (nt < ntiles) load_tile(nt % ATT_NST, k0 + nt * ATT_KT);
      cp_async_commit();
    }
    if (wrow >= nrows) continue;
    const ET* kst = ksm + (it % ATT_NST) * 2 * ATT_KT * XS;
    const ET* vst = kst + ATT_KT * XS;
    // S = Q K^T for 16 rows x 32 keys
    float sc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll 4
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t af[4];
      ldmatrix_x4(af, qsm + qa_row * XS + ks * 16 + qa_col);
#pragma unroll
      for (int jp = 0; jp < 2; ++jp) {
        uint32_t bf[4];
        ldmatrix_x4(bf, kst + (jp * 16 + kb_key) * XS + ks * 16 + kb_col);
        mma16816<ET>(sc[2 * jp], af, bf[0], bf[1]);
        mma16816<ET>(sc[2 * jp + 1], af, bf[2], bf[3]);
      }
    }
    // scale, mask, online softmax
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int key = t0 + j * 8 + 2 * tig + (r & 1);
        const int h2 = r >> 1;
        const bool ok = key < k1 && key <= smax[h2] && key >= smin[h2];
        const float s = ok ? sc[j][r] * a.scale : -INFINITY;
        sc[j][r] = s;
        tmax[h2] = fmaxf(tmax[h2], s);
      }
    float corr[2];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      tmax[h2] = fmaxf(tmax[h2], __shfl_xor_sync(0xffffffffu, tmax[h2], 1));
      tmax[h2] = fmaxf(tmax[h2], __shfl_xor_sync(0xffffffffu, tmax[h2], 2));
      const float mn = fmaxf(m_run[h2], tmax[h2]);
      corr[h2] = (m_run[h2] == -INFINITY) ? 0.f : __expf(m_run[h2] - mn);
      m_run[h2] = mn;
    }
    float psum[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int h2 = r >> 1;
        const float p = (sc[j][r] == -INFINITY) ? 0.f : __expf(sc[j][r] - m_run[h2]);
        sc[j][r] = p;
        psum[h2] += p;
      }
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      psum[h2] += __shfl_xor_sync(0xffffffffu, psum[h2], 1);
      psum[h2] += __shfl_xor_sync(0xffffffffu, psum[h2], 2);
      l_run[h2] = l_run[h2] * corr[h2] + psum[h2];
    }
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      o[j][0] *= corr[0]; o[j][1] *= corr[0];
      o[j][2] *= corr[1]; o[j][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t pf[4];
      pf[0] = pack2(sc[2 * kk][0], sc[2 * kk][1], f16);
      pf[1] = pack2(sc[2 * kk][2], sc[2 * kk][3], f16);
      pf[2] = pack2(sc[2 * kk + 1][0], sc[2 * kk + 1][1], f16);
      pf[3] = pack2(sc[2 * kk + 1][2], sc[2 * kk + 1][3], f16);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t vf[4];
        ldmatrix_x4_trans(vf, vst + (kk * 16 + vb_key) * XS + dp * 16 + vb_col);
        mma16816<ET>(o[2 * dp], pf, vf[0], vf[1]);
        mma16816<ET>(o[2 * dp + 1], pf, vf[2], vf[3]);
      }
    }
  }
  if (wrow >= nrows) return;
  // partials
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2) {
    const int lr = wrow + gid + 8 * h2;
    if (lr >= nrows) continue;
    const int rr = row0 + lr;
    const int h = kvh * G + rr / a.S, s = rr % a.S;
    const int64_t base = ((static_cast<int64_t>(split) * a.B + b) * a.H + h) * a.S + s;
    float* op = a.opart + base * D;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const int d = j * 8 + 2 * tig;
      *reinterpret_cast<float2*>(op + d) = make_float2(o[j][2 * h2], o[j][2 * h2 + 1]);
    }
    if (tig == 0) {
      a.ml[base * 2] = m_run[h2];
      a.ml[base * 2 + 1] = l_run[h2];
    }
  }
}

// out element (b, h, s, d) at out + b*ob + h*oh + s*os + d; gate (optional) likewise.
// One CTA per (b, h, s): warp 0 turns the splits' (max, sum) pairs into per-split
// weights exp(m - M) (0 for a split with no visible key) and the total L; then every
// thread sums its output columns over the splits in split order.
constexpr int ATT_MAXSPLIT = 64;

template <typename ET, int D>
__global__ void attn_combine_kernel(const float* __restrict__ opart, const float* __restrict__ ml,
                                    ET* __restrict__ out, int64_t ob, int64_t oh, int64_t os,
                                    const ET* __restrict__ gate, int64_t gb, int64_t gh, int64_t gs,
                                    const int32_t* __restrict__ qposv, int qpos_scalar, int B, int H,
                                    int S, int kc) {
  __shared__ float s_w[ATT_MAXSPLIT];
  __shared__ float s_l;
  const int s = blockIdx.x % S, h = (blockIdx.x / S) % H, b = blockIdx.x / (S * H);
  // before the wait: the positions and the output gate, which the split kernel (the
  // predecessor) does not write; with dim <= 256 every thread owns one column
  const int qpos = qposv ? qposv[b] : qpos_scalar;
  constexpr bool ONE = D <= 256;
  float gpre = 0.f;
  if (ONE && gate && threadIdx.x < D) gpre = rnd<ET>(sigmoid_f(to_f(gate[b * gb + h * gh + s * gs + threadIdx.x])));
  pdl_wait();
  pdl_trigger();
  const int nsp = (qpos + S + kc - 1) / kc;
  const int64_t row = (static_cast<int64_t>(b) * H + h) * S + s;   // row index within one split
  const int64_t split_stride = static_cast<int64_t>(B) * H * S;
  // the first PRE splits' partials of this thread's column, requested now, while warp 0
  // turns the (max, sum) pairs into weights: one load round trip instead of several
  constexpr int PRE = 32;
  float pre[PRE];
  if (ONE) {
    const float* op = opart + row * D + threadIdx.x;
#pragma unroll
    for (int sp = 0; sp < PRE; ++sp) pre[sp] = (sp < nsp && threadIdx.x < D) ? op[sp * split_stride * D] : 0.f;
  }
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float m[2], l[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int sp = lane + 32 * u;
      m[u] = -INFINITY; l[u] = 0.f;
      if (sp < nsp) { m[u] = ml[(sp * split_stride + row) * 2]; l[u] = ml[(sp * split_stride + row) * 2 + 1]; }
    }
    const float M = warp_max(fmaxf(m[0], m[1]));
    float L = 0.f;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int sp = lane + 32 * u;
      const float w = (m[u] == -INFINITY) ? 0.f : __expf(m[u] - M);
      if (sp < nsp) s_w[sp] = w;
      L += w * l[u];
    }
    L = warp_sum(L);
    if (lane == 0) s_l = L;
  }
  __syncthreads();
  const float L = s_l;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    const float* op = opart + row * D + d;
    int sp0 = 0;
    if (ONE) {   // d == threadIdx.x: the prefetched splits first, in split order
#pragma unroll
      for (int sp = 0; sp < PRE; ++sp) {
        const float w = sp < nsp ? s_w[sp] : 0.f;
        if (w != 0.f) acc += w * pre[sp];
      }
      sp0 = PRE;
    }
#pragma unroll 8
    for (int sp = sp0; sp < nsp; ++sp) {
      const float w = s_w[sp];
      const float v = op[sp * split_stride * D];
      if (w != 0.f) acc += w * v;
    }
    float y = rnd<ET>(acc / L);
    if (gate) y = rnd<ET>(y * (ONE ? gpre : rnd<ET>(sigmoid_f(to_f(gate[b * gb + h * gh + s * gs + d])))));
    out[b * ob + h * oh + s * os + d] = from_f<ET>(y);
  }
}

// q/k RMSNorm + RoPE + KV append.  One CTA per (token, head slot): slots [0, H) are query
// heads, [H, H + Hkv) key heads (which also copy their value head).
constexpr int ATT_PREP_THREADS = 128;

template <int D>
__global__ void __launch_bounds__(ATT_PREP_THREADS) attn_prep_kernel(
    const __nv_bfloat16* __restrict__ qkv, int64_t ldq, const __nv_bfloat16* __restrict__ qn_w,
    const __nv_bfloat16* __restrict__ kn_w, float eps, float theta, int rot, const int32_t* __restrict__ qpos,
    const int32_t* __restrict__ pages, int max_pages, int P, __nv_bfloat16* __restrict__ kc,
    __nv_bfloat16* __restrict__ vc, __nv_bfloat16* __restrict__ qout, int S, int H, int Hkv) {
  constexpr int NPT = (D + ATT_PREP_THREADS - 1) / ATT_PREP_THREADS;   // columns per thread
  __shared__ float red[32];
  __shared__ float xr[D];
  const int t = blockIdx.x;  // token row b*S + s
  const int b = t / S, s = t % S;
  const int slot = blockIdx.y;
  const bool is_q = slot < H;
  const int head = is_q ? slot : slot - H;
  // before the wait: the norm weight, the rotary factors and the cache page, none of
  // which the projection (the predecessor) writes
  const __nv_bfloat16* gw = is_q ? qn_w : kn_w;
  const int pos = qpos[b] + s;
  const int half = rot / 2;
  float gpre[NPT], cpre[NPT], spre[NPT];
#pragma unroll
  for (int j = 0; j < NPT; ++j) {
    const int d = threadIdx.x + j * ATT_PREP_THREADS;
    gpre[j] = cpre[j] = spre[j] = 0.f;
    if (d < D) gpre[j] = rbf(__bfloat162float(gw[d]) + 1.f);  // zero-centred weight + 1
    if (d < rot) {
      const int i = d % half;
      const float inv_freq = 1.0f / powf(theta, static_cast<float>(2 * i) / rot);
      const float ang = static_cast<float>(pos) * inv_freq;
      cpre[j] = rbf(cosf(ang));
      spre[j] = rbf(sinf(ang));
    }
  }
  const int page = is_q ? 0 : pages[b * max_pages + pos / P];
  pdl_wait();   // qkv comes from the predecessor (the projection)
  pdl_trigger();
  const __nv_bfloat16* src = is_q ? qkv + t * ldq + head * 2 * D : qkv + t * ldq + H * 2 * D + head * D;
  float xv[NPT];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NPT; ++j) {
    const int d = threadIdx.x + j * ATT_PREP_THREADS;
    xv[j] = d < D ? __bfloat162float(src[d]) : 0.f;
    ss += xv[j] * xv[j];
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / D + eps);
#pragma unroll
  for (int j = 0; j < NPT; ++j) {
    const int d = threadIdx.x + j * ATT_PREP_THREADS;
    if (d < D) xr[d] = rbf(rbf(xv[j] * inv) * gpre[j]);
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < NPT; ++j) {
    const int d = threadIdx.x + j * ATT_PREP_THREADS;
    if (d >= D) continue;
    float y = xr[d];
    if (d < rot) {
      const float other = d < half ? -xr[d + half] : xr[d - half];
      y = rbf(rbf(xr[d] * cpre[j]) + rbf(other * spre[j]));
    }
    if (is_q) {
      qout[((static_cast<int64_t>(b) * H + head) * S + s) * D + d] = __float2bfloat16_rn(y);
    } else {
      const int64_t off = ((static_cast<int64_t>(page) * Hkv + head) * P + pos % P) * D + d;
      kc[off] = __float2bfloat16_rn(y);
      vc[off] = qkv[t * ldq + H * 2 * D + Hkv * D + head * D + d];
    }
  }
}

// -------------------------------------------------------------------------- host side
struct SplitPlan {
  int kc, nsplit, rowgroups;
};

static SplitPlan plan_splits(int B, int H, int Hkv, int S, int max_len) {
  SplitPlan p;
  const int R = (H / Hkv) * S;
  p.rowgroups = (R + ATT_MAXROWS - 1) / ATT_MAXROWS;
  const int units = B * Hkv * p.rowgroups;
  int target = (296 + units - 1) / units;
  const int max_tiles = (max_len + ATT_KT - 1) / ATT_KT;
  if (target > 64) target = 64;
  if (target > max_tiles) target = max_tiles;
  if (target < 1) target = 1;
  int kc = (max_len + target - 1) / target;
  if (kc < ATT_MIN_KC) kc = ATT_MIN_KC;
  kc = (kc + ATT_KT - 1) / ATT_KT * ATT_KT;
  p.kc = kc;
  p.nsplit = (max_len + kc - 1) / kc;
  return p;
}

template <typename ET, int D>
static int launch_attn(AttnArgs<ET> a, ET* out, int64_t ob, int64_t oh, int64_t os, const ET* gate,
                       int64_t gb, int64_t gh, int64_t gs, cudaStream_t st) {
  const int G = a.H / a.Hkv;
  const int R = G * a.S;
  const int rows_cta = R < ATT_MAXROWS ? R : ATT_MAXROWS;
  const int warps = (rows_cta + 15) / 16;
  const size_t smem = (static_cast<size_t>(ATT_MAXROWS) + ATT_NST * 2 * ATT_KT) * (D + 8) * sizeof(ET) +
                     ATT_PGCAP * sizeof(int);
  a.pgcap = ATT_PGCAP;
  a.plog2 = (a.P > 0 && (a.P & (a.P - 1)) == 0) ? __builtin_ctz(static_cast<unsigned>(a.P)) : -1;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    err = cudaFuncSetAttribute(attn_split_kernel<ET, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  if (err != cudaSuccess) return cuda_status(err, "attention smem attribute");
  if (a.nsplit > ATT_MAXSPLIT) return fail(QW_ERR_UNSUPPORTED, "attention: %d key splits", a.nsplit);
  QW_LAUNCH_PDL("attention split", attn_split_kernel<ET, D>, dim3(a.nsplit, a.Hkv * a.rowgroups, a.B),
                dim3(warps * 32), smem, st, a);
  QW_LAUNCH_PDL("attention combine", attn_combine_kernel<ET, D>, dim3(a.B * a.H * a.S), dim3(D < 256 ? D : 256), 0,
                st, static_cast<const float*>(a.opart), static_cast<const float*>(a.ml), out, ob, oh, os, gate, gb,
                gh, gs, a.qpos, a.qpos_scalar, a.B, a.H, a.S, a.kc);
  return QW_OK;
}

template <typename ET>
static int dispatch_attn(int D, const AttnArgs<ET>& a, ET* out, int64_t ob, int64_t oh, int64_t os,
                         const ET* gate, int64_t gb, int64_t gh, int64_t gs, cudaStream_t st) {
  switch (D) {
    case 32: return launch_attn<ET, 32>(a, out, ob, oh, os, gate, gb, gh, gs, st);
    case 64: return launch_attn<ET, 64>(a, out, ob, oh, os, gate, gb, gh, gs, st);
    case 128: return launch_attn<ET, 128>(a, out, ob, oh, os, gate, gb, gh, gs, st);
    case 256: return launch_attn<ET, 256>(a, out, ob, oh, os, gate, gb, gh, gs, st);
  }
  return fail(QW_ERR_UNSUPPORTED, "attention: head dim %d not built (32, 64, 128, 256)", D);
}

}  // namespace qw

using namespace qw;

extern "C" int64_t qw_attn_workspace_bytes(int64_t batch, int64_t heads, int64_t kv_heads, int64_t seq,
                                           int64_t dim, int64_t max_len) {
  if (batch < 1 || heads < 1 || kv_heads < 1 || seq < 1 || dim < 1 || max_len < seq) return -1;
  SplitPlan p = plan_splits(static_cast<int>(batch), static_cast<int>(heads), static_cast<int>(kv_heads),
                            static_cast<int>(seq), static_cast<int>(max_len));
  return static_cast<int64_t>(p.nsplit) * batch * heads * seq * (dim + 2) * 4;
}

extern "C" int qw_attention(const void* q, const void* k, const void* v, void* out, int dtype, int64_t batch,
                            int64_t heads, int64_t kv_heads, int64_t seq, int64_t total, int64_t dim,
                            int64_t query_start, float scale, void* workspace, void* stream) {
  QW_CHECK_ARG(q && k && v && out && workspace, "attention: null pointer");
  QW_CHECK_ARG(batch >= 1 && heads >= 1 && kv_heads >= 1 && heads % kv_heads == 0 && seq >= 1 &&
                   query_start >= 0 && query_start + seq == total && scale > 0.f && batch < 65536,
               "attention requires causal append-only GQA [B,H,S,D] inputs");
  QW_CHECK_ARG(dtype == QW_BF16 || dtype == QW_F16, "attention: bf16 or fp16 required");
  SplitPlan p = plan_splits(static_cast<int>(batch), static_cast<int>(heads), static_cast<int>(kv_heads),
                            static_cast<int>(seq), static_cast<int>(total));
  const int64_t S = seq, D = dim, T = total;
  cudaStream_t st = as_stream(stream);
  float* opart = static_cast<float*>(workspace);
  float* ml = opart + static_cast<int64_t>(p.nsplit) * batch * heads * seq * dim;
#define QW_ATT(ET)                                                                                  \
  do {                                                                                              \
    AttnArgs<ET> a{};                                                                               \
    a.q = static_cast<const ET*>(q); a.qb = heads * S * D; a.qh = S * D; a.qs = D;                 \
    a.k = static_cast<const ET*>(k); a.v = static_cast<const ET*>(v);                              \
    a.pages = nullptr; a.max_pages = 1; a.P = static_cast<int>(T);                                  \
    a.qpos = nullptr; a.qpos_scalar = static_cast<int>(query_start);                                \
    a.B = static_cast<int>(batch); a.H = static_cast<int>(heads); a.Hkv = static_cast<int>(kv_heads); \
    a.S = static_cast<int>(seq); a.kc = p.kc; a.nsplit = p.nsplit; a.rowgroups = p.rowgroups;       \
    a.scale = scale; a.opart = opart; a.ml = ml;                                                    \
    return dispatch_attn<ET>(static_cast<int>(dim), a, static_cast<ET*>(out), heads * S * D, S * D, D, \
                             nullptr, 0, 0, 0, st);                                                 \
  } while (0)
  if (dtype == QW_BF16) QW_ATT(__nv_bfloat16);
  QW_ATT(__half);
#undef QW_ATT
}

extern "C" int qw_attn_prep(const void* qkv, int64_t ldq, const void* q_norm_w, const void* k_norm_w, float eps,
                            float rope_theta, int32_t rotary_dim, const int32_t* qpos, const int32_t* pages,
                            int32_t max_pages, int32_t page_size, void* k_cache, void* v_cache, void* q_out,
                            int64_t batch, int64_t seq, int64_t heads, int64_t kv_heads, int64_t dim,
                            void* stream) {
  QW_CHECK_ARG(qkv && q_norm_w && k_norm_w && qpos && pages && k_cache && v_cache && q_out,
               "attn_prep: null pointer");
  QW_CHECK_ARG(batch >= 1 && seq >= 1 && heads >= 1 && kv_heads >= 1 && page_size >= 1 && max_pages >= 1 &&
                   rotary_dim >= 2 && rotary_dim % 2 == 0 && rotary_dim <= dim &&
                   ldq >= heads * 2 * dim + 2 * kv_heads * dim,
               "attn_prep: invalid shape");
  const dim3 grid(static_cast<unsigned>(batch * seq), static_cast<unsigned>(heads + kv_heads));
  cudaStream_t st = as_stream(stream);
#define QW_PREP(DD)                                                                                     \
  QW_LAUNCH_PDL("attn_prep", attn_prep_kernel<DD>, grid, dim3(ATT_PREP_THREADS), 0, st,                              \
      static_cast<const __nv_bfloat16*>(qkv), ldq, static_cast<const __nv_bfloat16*>(q_norm_w),        \
      static_cast<const __nv_bfloat16*>(k_norm_w), eps, rope_theta, rotary_dim, qpos, pages, max_pages, \
      page_size, static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache),            \
      static_cast<__nv_bfloat16*>(q_out), static_cast<int>(seq), static_cast<int>(heads),              \
      static_cast<int>(kv_heads))
  switch (dim) {
    case 64: QW_PREP(64); break;
    case 128: QW_PREP(128); break;
    case 256: QW_PREP(256); break;
    default: return fail(QW_ERR_UNSUPPORTED, "attn_prep: head dim %lld not built", static_cast<long long>(dim));
  }
#undef QW_PREP
  QW_LAUNCH_CHECK("attn_prep");
  return QW_OK;
}

static int attn_paged_entry(const void* q, const void* k_cache, const void* v_cache, const int32_t* pages,
                            int32_t max_pages, int32_t page_size, const int32_t* qpos, int64_t max_len,
                            const void* gate, int64_t ldg, void* out, int64_t batch, int64_t seq, int64_t heads,
                            int64_t kv_heads, int64_t dim, float scale, void* workspace, void* stream, int block_full,
                            int window);

extern "C" int qw_attn_paged(const void* q, const void* k_cache, const void* v_cache, const int32_t* pages,
                             int32_t max_pages, int32_t page_size, const int32_t* qpos, int64_t max_len,
                             const void* gate, int64_t ldg, void* out, int64_t batch, int64_t seq, int64_t heads,
                             int64_t kv_heads, int64_t dim, float scale, void* workspace, void* stream) {
  return attn_paged_entry(q, k_cache, v_cache, pages, max_pages, page_size, qpos, max_len, gate, ldg, out, batch, seq,
                          heads, kv_heads, dim, scale, workspace, stream, 0, 0);
}

extern "C" int qw_attn_paged_masked(const void* q, const void* k_cache, const void* v_cache, const int32_t* pages,
                                    int32_t max_pages, int32_t page_size, const int32_t* qpos, int64_t max_len,
                                    void* out, int64_t batch, int64_t seq, int64_t heads, int64_t kv_heads,
                                    int64_t dim, float scale, int block_full, int32_t window, void* workspace,
                                    void* stream) {
  QW_CHECK_ARG(window >= 0 && (block_full == 0 || block_full == 1), "attn_paged_masked: invalid mask");
  return attn_paged_entry(q, k_cache, v_cache, pages, max_pages, page_size, qpos, max_len, nullptr, 0, out, batch,
                          seq, heads, kv_heads, dim, scale, workspace, stream, block_full, window);
}

static int attn_paged_entry(const void* q, const void* k_cache, const void* v_cache, const int32_t* pages,
                            int32_t max_pages, int32_t page_size, const int32_t* qpos, int64_t max_len,
                            const void* gate, int64_t ldg, void* out, int64_t batch, int64_t seq, int64_t heads,
                            int64_t kv_heads, int64_t dim, float scale, void* workspace, void* stream, int block_full,
                            int window) {
  QW_CHECK_ARG(q && k_cache && v_cache && pages && qpos && out && workspace, "attn_paged: null pointer");
  QW_CHECK_ARG(batch >= 1 && seq >= 1 && heads >= 1 && kv_heads >= 1 && heads % kv_heads == 0 && max_len >= seq &&
                   page_size >= 1 && max_pages * static_cast<int64_t>(page_size) >= max_len && scale > 0.f,
               "attn_paged: invalid shape");
  SplitPlan p = plan_splits(static_cast<int>(batch), static_cast<int>(heads), static_cast<int>(kv_heads),
                            static_cast<int>(seq), static_cast<int>(max_len));
  AttnArgs<__nv_bfloat16> a{};
  const int64_t S = seq, D = dim, H = heads;
  a.q = static_cast<const __nv_bfloat16*>(q); a.qb = H * S * D; a.qh = S * D; a.qs = D;
  a.k = static_cast<const __nv_bfloat16*>(k_cache); a.v = static_cast<const __nv_bfloat16*>(v_cache);
  a.pages = pages; a.max_pages = max_pages; a.P = page_size;
  a.qpos = qpos; a.qpos_scalar = 0;
  a.B = static_cast<int>(batch); a.H = static_cast<int>(heads); a.Hkv = static_cast<int>(kv_heads);
  a.S = static_cast<int>(seq); a.kc = p.kc; a.nsplit = p.nsplit; a.rowgroups = p.rowgroups;
  a.scale = scale;
  a.block_full = block_full;
  a.window = window;
  a.opart = static_cast<float*>(workspace);
  a.ml = a.opart + static_cast<int64_t>(p.nsplit) * batch * heads * seq * dim;
  // out [B*S, H*D]; gate element (b, h, s, d) at gate + (b*S + s)*ldg + h*2D + d
  return dispatch_attn<__nv_bfloat16>(static_cast<int>(dim), a, static_cast<__nv_bfloat16*>(out), S * H * D, D,
                                      H * D, static_cast<const __nv_bfloat16*>(gate), S * ldg, 2 * D, ldg,
                                      as_stream(stream));
}

// ------------------------------------------------------------------ allocation-free variant
// qw_attention_noalloc: qw_attention with its split-K scratch taken from a fixed array
// in this library's device memory instead of a caller-supplied workspace, for callers
// that cannot allocate device memory (a host runtime with its own pool and no hook for
// per-call scratch, a driver thread that must not call cudaMalloc because it would
// synchronise the device).  The array is a file-scope __device__ variable: every GPU
// that loads this module holds QW_ATTN_NOALLOC_SCRATCH_BYTES of it until the process
// exits.  Host code never uses the array's name as a pointer (on the host it is only a
// stand-in symbol); the device address comes from cudaGetSymbolAddress, looked up once
// per device, with that device current, on the first call made on it.
namespace qw {

static __device__ __align__(256) float g_attn_noalloc_scratch[QW_ATTN_NOALLOC_SCRATCH_BYTES / sizeof(float)];

constexpr int NOALLOC_MAX_DEVICES = 64;
static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};

// Device address of the scratch array on the current device (looked up on first use).
static int noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_status(err, "attention_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES)
    return fail(QW_ERR_UNSUPPORTED, "attention_noalloc: device %d beyond the %d this build tracks", dev,
                NOALLOC_MAX_DEVICES);
  std::lock_guard<std::mutex> guard(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (err != cudaSuccess) return cuda_status(err, "attention_noalloc: cudaGetSymbolAddress of the scratch");
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return QW_OK;
}

}  // namespace qw

extern "C" int qw_attention_noalloc(const void* q, const void* k, const void* v, void* out, int dtype,
                                    int64_t batch, int64_t heads, int64_t kv_heads, int64_t seq, int64_t total,
                                    int64_t dim, int64_t query_start, float scale, void* stream) {
  QW_CHECK_ARG(q && k && v && out, "attention_noalloc: null pointer");
  QW_CHECK_ARG(batch >= 1 && heads >= 1 && kv_heads >= 1 && heads % kv_heads == 0 && seq >= 1 &&
                   query_start >= 0 && query_start + seq == total && scale > 0.f && batch < 65536,
               "attention_noalloc requires causal append-only GQA [B,H,S,D] inputs");
  QW_CHECK_ARG(dtype == QW_BF16 || dtype == QW_F16, "attention_noalloc: bf16 or fp16 required");
  if (dim != 32 && dim != 64 && dim != 128 && dim != 256)
    return fail(QW_ERR_UNSUPPORTED, "attention_noalloc: head dim %lld not built (32, 64, 128, 256)",
                static_cast<long long>(dim));
  SplitPlan p = plan_splits(static_cast<int>(batch), static_cast<int>(heads), static_cast<int>(kv_heads),
                            static_cast<int>(seq), static_cast<int>(total));
  // the same sizing as a caller workspace of qw_attention, so the bound cannot drift
  // from the split plan or the opart / ml layout below
  const int64_t need = qw_attn_workspace_bytes(batch, heads, kv_heads, seq, dim, total);
  QW_CHECK_ARG(need >= 0, "attention_noalloc: no workspace size for this shape");
  QW_CHECK_ARG(need <= static_cast<int64_t>(QW_ATTN_NOALLOC_SCRATCH_BYTES),
               "attention_noalloc: this shape needs %lld scratch bytes, the static scratch holds %lld "
               "(use qw_attention with a caller workspace)",
               static_cast<long long>(need), static_cast<long long>(QW_ATTN_NOALLOC_SCRATCH_BYTES));
  float* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != QW_OK) return rc;
  // Nothing in the scratch has to start at zero: the split kernel writes every
  // (split, row) partial and max/sum pair that the combine kernel then reads, so the
  // previous call's contents are never observed.
  const int64_t S = seq, D = dim, T = total;
  cudaStream_t st = as_stream(stream);
  float* opart = scratch;
  float* ml = opart + static_cast<int64_t>(p.nsplit) * batch * heads * seq * dim;
#define QW_ATT_NA(ET)                                                                               \
  do {                                                                                              \
    AttnArgs<ET> a{};                                                                               \
    a.q = static_cast<const ET*>(q); a.qb = heads * S * D; a.qh = S * D; a.qs = D;                 \
    a.k = static_cast<const ET*>(k); a.v = static_cast<const ET*>(v);                              \
    a.pages = nullptr; a.max_pages = 1; a.P = static_cast<int>(T);                                  \
    a.qpos = nullptr; a.qpos_scalar = static_cast<int>(query_start);                                \
    a.B = static_cast<int>(batch); a.H = static_cast<int>(heads); a.Hkv = static_cast<int>(kv_heads); \
    a.S = static_cast<int>(seq); a.kc = p.kc; a.nsplit = p.nsplit; a.rowgroups = p.rowgroups;       \
    a.scale = scale; a.opart = opart; a.ml = ml;                                                    \
    return dispatch_attn<ET>(static_cast<int>(dim), a, static_cast<ET*>(out), heads * S * D, S * D, D, \
                             nullptr, 0, 0, 0, st);                                                 \
  } while (0)
  if (dtype == QW_BF16) QW_ATT_NA(__nv_bfloat16);
  QW_ATT_NA(__half);
#undef QW_ATT_NA
}
