// Gated DeltaNet kernels.
//
//  * qw_gated_delta_rule — the fused-ops ABI operator (reference/fused_ops.py:59-107):
//    sequential recurrence, one CTA per (sequence, head), state in shared memory.
//  * qw_gdn_verify / qw_gdn_commit — the block-verify form.  One thread-block cluster
//    per (sequence, value head); each CTA of the cluster owns Dv/VSPLIT state columns
//    and keeps them in registers (8 threads per column, Dk/8 rows each) across the
//    block's tokens (a prefill chunk longer than QW_MAX_BLOCK is taken in sub-blocks of
//    QW_MAX_BLOCK, the state staying in registers and each full sub-block's last inputs
//    becoming the next one's conv tail).  The prologue fuses conv_state_update + causal_conv1d + SiLU
//    (fused/model.py:232-239; the head's q|k channels split over the cluster's CTAs and
//    pushed to all of them through distributed shared memory), the q/k L2 norm and the
//    gate math (:243-253); the
//    epilogue fuses the gated RMSNorm x SiLU(z) (:219-225), with the row sum of squares
//    exchanged through distributed shared memory.  Verify never writes the recurrent
//    state: commit recomputes the first r tokens from the same inputs with the same
//    arithmetic, so the committed state equals the verify's state after r tokens.
#include <cooperative_groups.h>

#include "qw_common.cuh"

namespace cg = cooperative_groups;

namespace qw {

using GdnLayer = qw_gdn_layer;
using GdnDims = qw_gdn_dims;

// =============================================================== fused-ops operator
template <typename Tin, typename Tst>
__global__ void gdn_rule_kernel(const Tin* __restrict__ q, const Tin* __restrict__ k,
                                const Tin* __restrict__ v, const Tin* __restrict__ g,
                                const Tin* __restrict__ beta, const Tst* __restrict__ s0,
                                const int16_t* __restrict__ eff_len, Tin* __restrict__ core,
                                Tst* __restrict__ s_out, int seq, int heads, int dk, int dv,
                                int use_l2) {
  extern __shared__ float smem[];
  float* S = smem;                 // [dk][dv]
  float* qs = S + dk * dv;         // [dk]
  float* ks = qs + dk;             // [dk]
  float* red = ks + dk;            // [64]
  const int h = blockIdx.x, b = blockIdx.y;
  const int64_t bh = static_cast<int64_t>(b) * heads + h;
  for (int i = threadIdx.x; i < dk * dv; i += blockDim.x) S[i] = to_f(s0[bh * dk * dv + i]);
  const int len = eff_len[b];
  const float qscale = rsqrtf(static_cast<float>(dk));
  for (int t = 0; t < seq; ++t) {
    const int64_t row = (static_cast<int64_t>(b) * seq + t) * heads + h;
    __syncthreads();
    float sq = 0.f, sk = 0.f;
    for (int i = threadIdx.x; i < dk; i += blockDim.x) {
      float a = to_f(q[row * dk + i]), c = to_f(k[row * dk + i]);
      qs[i] = a;
      ks[i] = c;
      sq += a * a;
      sk += c * c;
    }
    sq = block_sum(sq, red);
    sk = block_sum(sk, red + 32);
    const float iq = use_l2 ? rsqrtf(sq + 1e-6f) : 1.f;
    const float ik = use_l2 ? rsqrtf(sk + 1e-6f) : 1.f;
    const bool valid = t < len;
    const float decay = __expf(to_f(g[row]));
    const float bt = to_f(beta[row]);
    for (int c = threadIdx.x; c < dv; c += blockDim.x) {
      float o = 0.f;
      if (valid) {
        float pred = 0.f;
        for (int i = 0; i < dk; ++i) {
          float sv = S[i * dv + c] * decay;
          S[i * dv + c] = sv;
          pred = fmaf(sv, ks[i] * ik, pred);
        }
        const float delta = (to_f(v[row * dv + c]) - pred) * bt;
        for (int i = 0; i < dk; ++i) {
          float sv = fmaf(ks[i] * ik, delta, S[i * dv + c]);
          S[i * dv + c] = sv;
          o = fmaf(sv, qs[i] * iq * qscale, o);
        }
      }
      core[row * dv + c] = from_f<Tin>(o);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < dk * dv; i += blockDim.x) s_out[bh * dk * dv + i] = from_f<Tst>(S[i]);
}

// =============================================================== block verify / commit
constexpr int KSPLIT = 8;  // threads per state column

template <int DK, int DV, int VSPLIT>
struct GdnTile {
  static constexpr int COLS = DV / VSPLIT;         // state columns per CTA
  static constexpr int THREADS = COLS * KSPLIT;    // 128 for COLS = 32
  static constexpr int ROWS = DK / KSPLIT;         // state rows per thread
};

// Shared-memory layout of one CTA (floats).
template <int DK, int DV, int VSPLIT>
struct GdnSmem {
  static constexpr int COLS = DV / VSPLIT;
  float q[QW_MAX_BLOCK][DK];
  float k[QW_MAX_BLOCK][DK];
  float v[QW_MAX_BLOCK][COLS];
  float o[QW_MAX_BLOCK][COLS];
  float opart[QW_MAX_BLOCK][COLS][KSPLIT];   // per-thread partial outputs, reduced after the recurrence
  float g[QW_MAX_BLOCK];
  float beta[QW_MAX_BLOCK];
  float sumsq[VSPLIT][QW_MAX_BLOCK];   // per-token sums of squares of each cluster rank
  float total[QW_MAX_BLOCK];
  // the block's projections of this CTA's channels: q [0, DK), k [DK, 2DK), v [2DK, 2DK+COLS)
  __align__(16) __nv_bfloat16 xin[QW_MAX_BLOCK][2 * DK + COLS];
  __align__(16) __nv_bfloat16 zin[QW_MAX_BLOCK][COLS];   // output gate inputs
};

// Position in shared memory of q/k element j: the thread owning state rows
// [kq * ROWS, (kq + 1) * ROWS) reads its elements i..i+3 (i a multiple of 4) as one
// 16-byte vector at (i / 4) * 4 * KSPLIT + 4 * kq, so the KSPLIT threads of a column
// read consecutive vectors (no bank conflicts).
template <int DK>
__device__ __forceinline__ int kperm(int j) {
  constexpr int ROWS = DK / KSPLIT;
  const int kq = j / ROWS, i = j % ROWS;
  return (i / 4) * (4 * KSPLIT) + kq * 4 + (i % 4);
}

// conv + SiLU of one channel over the block's tokens, rounded to bf16 after the conv and
// after the SiLU (the reference's activation tensors, fused/model.py:238-239).  hist /
// w hold the channel's conv tail and taps, the block inputs come from shared memory
// (src[t * sstride]).  Every row of the block buffer is computed (rows past the block's
// tokens hold stale, in-bounds values) so the unrolled tokens interleave; the caller
// stores the real ones.
constexpr int GDN_CONV_K = 4;  // conv taps of the block kernels

__device__ __forceinline__ void conv_channel(const float (&hist)[GDN_CONV_K - 1], const float (&w)[GDN_CONV_K],
                                             const __nv_bfloat16* src, int sstride, float (&y)[QW_MAX_BLOCK]) {
  constexpr int K = GDN_CONV_K;
  float win[K];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) win[j] = hist[j];
#pragma unroll
  for (int t = 0; t < QW_MAX_BLOCK; ++t) {
    win[K - 1] = __bfloat162float(src[t * sstride]);
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) acc = fmaf(win[j], w[j], acc);
    y[t] = rbf(silu_f(rbf(acc)));
#pragma unroll
    for (int j = 0; j < K - 1; ++j) win[j] = win[j + 1];
  }
}

// Four CTAs per SM (64 registers, no spills; the shared memory allows four): at batch 8
// and up the grid is several waves of clusters, and residency sets the throughput.
template <int DK, int DV, int VSPLIT, bool COMMIT>
__global__ void __launch_bounds__(GdnTile<DK, DV, VSPLIT>::THREADS, 4)
    gdn_block_kernel(GdnDims d, const GdnLayer* __restrict__ layers, int layer0) {
  using Tile = GdnTile<DK, DV, VSPLIT>;
  constexpr int COLS = Tile::COLS, ROWS = Tile::ROWS, THREADS = Tile::THREADS;
  __shared__ GdnSmem<DK, DV, VSPLIT> sm;
  const int rank = blockIdx.x;          // column block within the head (cluster rank)
  const int h = blockIdx.y;             // value head
  const int b = blockIdx.z % d.batch;   // sequence within the batch
  const GdnLayer& L = layers[layer0 + blockIdx.z / d.batch];
  const int64_t slot = d.slots[b];
  // commit: the accepted counts come from the predecessor (accept); verify reads the
  // banks and the projections of earlier kernels first and waits before the gates
  if constexpr (COMMIT) {
    pdl_wait();
    pdl_trigger();
  }
  // tokens of the sequence: the block (verify), or its accepted prefix (commit); taken in
  // sub-blocks of QW_MAX_BLOCK with the state kept in registers (a prefill chunk is
  // longer than one verify block)
  const int total = COMMIT ? d.accepted[b] : d.seq;
  const int tid = threadIdx.x;
  const int col = tid / KSPLIT, kq = tid % KSPLIT;
  const int kh = h / (d.v_heads / d.k_heads);
  const int kw = d.k_heads * DK;
  const int vcol0 = rank * COLS;        // first state column of this CTA within the head

  if (COMMIT && total <= 0) return;     // nothing accepted (the whole cluster): the state stays S0

  // ---- state columns into registers (bank layout [slot][head][Dv][Dk], column-major);
  // issued first so their latency overlaps the staging below
  float st[ROWS];
  float* scol = L.state + ((slot * d.v_heads + h) * DV + vcol0 + col) * static_cast<int64_t>(DK) + kq * ROWS;
#pragma unroll
  for (int i = 0; i < ROWS; i += 4) {
    float4 v4 = *reinterpret_cast<const float4*>(scol + i);
    st[i] = v4.x; st[i + 1] = v4.y; st[i + 2] = v4.z; st[i + 3] = v4.w;
  }
  int t0 = 0, ntok = 0;   // the current sub-block: tokens [t0, t0 + ntok)
  // ---- stage a sub-block's projections of this CTA's channels (and z) in shared memory:
  // per token 8-element vectors of the q, k, v (and z) segments, all loads in flight at once
  auto stage = [&]() {
    const int vw = d.v_heads * DV;
    constexpr int QV = DK / 8, KV = DK / 8, VV = COLS / 8;
    constexpr int PER = QV + KV + VV + VV;
    const int64_t segq = kh * DK, segk = kw + kh * DK, segv = 2 * kw + h * DV + vcol0,
                  segz = 2 * kw + vw + h * DV + vcol0;
    for (int i = tid; i < ntok * PER; i += THREADS) {
      const int t = i / PER, v = i % PER;
      if (COMMIT && (v < QV || v >= QV + KV + VV)) continue;   // commit needs k and v only
      const __nv_bfloat16* rowp = L.proj + (static_cast<int64_t>(b) * d.seq + t0 + t) * d.ldp;
      const __nv_bfloat16* src;
      __nv_bfloat16* dst;
      if (v < QV) { src = rowp + segq + v * 8; dst = &sm.xin[t][v * 8]; }
      else if (v < QV + KV) { src = rowp + segk + (v - QV) * 8; dst = &sm.xin[t][DK + (v - QV) * 8]; }
      else if (v < QV + KV + VV) { src = rowp + segv + (v - QV - KV) * 8; dst = &sm.xin[t][2 * DK + (v - QV - KV) * 8]; }
      else { src = rowp + segz + (v - QV - KV - VV) * 8; dst = &sm.zin[t][(v - QV - KV - VV) * 8]; }
      cp_async16(dst, src, true);
    }
    cp_async_commit();
  };
  // ---- each thread's conv channels: tails and taps (older than the predecessor).  The
  // cluster's CTAs share the head's q and k: rank r convolves q|k channels
  // [r * QKR, (r + 1) * QKR) for all of them (verify: q then k; commit: k only), and
  // every CTA its own v columns.
  constexpr int K = GDN_CONV_K;
  constexpr int XS = 2 * DK + COLS;
  constexpr int CPT = (2 * DK / VSPLIT + COLS + THREADS - 1) / THREADS;  // channels per thread
  const int nq = COMMIT ? 0 : DK;
  const int qkr = (nq + DK) / VSPLIT;   // q|k channels this CTA convolves
  const int nch = qkr + COLS;
  float hreg[CPT][K - 1], wreg[CPT][K];
  int chan[CPT], src_col[CPT];
#pragma unroll
  for (int r = 0; r < CPT; ++r) {
    const int i = tid + r * THREADS;
    if (i < qkr) {
      const int j = rank * qkr + i + (DK - nq);   // 0 .. DK: q, DK .. 2DK: k
      chan[r] = j < DK ? kh * DK + j : kw + kh * DK + (j - DK);
      src_col[r] = j;
    } else {
      chan[r] = 2 * kw + h * DV + vcol0 + (i - qkr);
      src_col[r] = 2 * DK + (i - qkr);
    }
    if (i < nch) {
      const __nv_bfloat16* hist = L.conv_hist + (slot * d.channels + chan[r]) * (K - 1);
#pragma unroll
      for (int j = 0; j < K - 1; ++j) hreg[r][j] = __bfloat162float(hist[j]);
#pragma unroll
      for (int j = 0; j < K; ++j) wreg[r][j] = __bfloat162float(L.conv_w[chan[r] * K + j]);
    }
  }
  // per-thread constants of the gates and of the gated norm
  const float neg_a = -__expf(L.A_log[h]), dtb = L.dt_bias[h];
  const float norm_w = COMMIT ? 0.f : __bfloat162float(L.norm_w[vcol0 + tid % COLS]);
  // the phases before the recurrence; verify runs conv and the q/k norms, which need
  // only the projections (written before the launch ahead of this one), before its
  // wait, and the gates, which read that launch's output, after it
  auto conv_phase = [&]() {
    // ---- conv + SiLU for this CTA's share of q|k (into every cluster CTA) and its v
    // columns (taps and tails loaded above); q and k are stored with row j at kperm(j)
    // (see the recurrence).  A full sub-block's last K - 1 inputs are the next one's tail.
    if constexpr (VSPLIT > 1) cluster_wait();   // every peer CTA is running (arrived above)
#pragma unroll
    for (int r = 0; r < CPT; ++r) {
      const int i = tid + r * THREADS;
      if (i >= nch) continue;
      float y[QW_MAX_BLOCK];
      conv_channel(hreg[r], wreg[r], &sm.xin[0][src_col[r]], XS, y);
      if (ntok == QW_MAX_BLOCK) {
#pragma unroll
        for (int j = 0; j < K - 1; ++j)
          hreg[r][j] = __bfloat162float(sm.xin[QW_MAX_BLOCK - (K - 1) + j][src_col[r]]);
      }
      if (i < qkr) {
        const int j = src_col[r];
        float* dst = j < DK ? &sm.q[0][kperm<DK>(j)] : &sm.k[0][kperm<DK>(j - DK)];
#pragma unroll
        for (int pr = 0; pr < VSPLIT; ++pr) {
          float* to = dst;
          if constexpr (VSPLIT > 1) to = cg::this_cluster().map_shared_rank(dst, (rank + pr) % VSPLIT);
#pragma unroll
          for (int t = 0; t < QW_MAX_BLOCK; ++t)
            if (t < ntok) to[t * DK] = y[t];
        }
      } else {
#pragma unroll
        for (int t = 0; t < QW_MAX_BLOCK; ++t)
          if (t < ntok) sm.v[t][i - qkr] = y[t];
      }
    }
    // every CTA's share of q|k has landed everywhere
    if constexpr (VSPLIT > 1) cg::this_cluster().sync();
  };
  auto l2_phase = [&]() {
    // ---- L2 norm of q and k per token (fused_ops.py:92-95); q also scaled by Dk^-1/2:
    // 8 threads per token, all tokens at once
    {
      static_assert(THREADS >= 8 * QW_MAX_BLOCK, "the l2 norm needs 8 threads per token");
      const int t = tid / 8, part = tid % 8;
      float sk = 0.f, sq = 0.f;
      if (t < ntok) {
#pragma unroll
        for (int i = part; i < DK; i += 8) {
          sk += sm.k[t][i] * sm.k[t][i];
          if (!COMMIT) sq += sm.q[t][i] * sm.q[t][i];
        }
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
        if (!COMMIT) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      }
      if (t < ntok) {
        const float ik = rsqrtf(sk + 1e-6f);
        const float iq = COMMIT ? 0.f : rsqrtf(sq + 1e-6f) * rsqrtf(static_cast<float>(DK));
#pragma unroll
        for (int i = part; i < DK; i += 8) {
          sm.k[t][i] *= ik;
          if (!COMMIT) sm.q[t][i] *= iq;
        }
      }
    }
  };
  auto gates_phase = [&]() {
    // ---- gates (fused/model.py:243-253, fp32)
    for (int t = tid; t < ntok; t += THREADS) {
      const int64_t row = static_cast<int64_t>(b) * d.seq + t0 + t;
      const float bl = L.ab[row * 2 * d.v_heads + h];
      const float al = L.ab[row * 2 * d.v_heads + d.v_heads + h];
      sm.beta[t] = sigmoid_f(bl);
      sm.g[t] = __expf(neg_a * softplus_f(al + dtb));   // the decay exp(g) of the recurrence
    }
  };
  const int vw = d.v_heads * DV;
  for (t0 = 0; t0 < total; t0 += QW_MAX_BLOCK) {
    ntok = min(QW_MAX_BLOCK, total - t0);
    // the conv outputs of q and k are pushed into the peer CTAs' shared memory; the
    // arrival here and the wait before those stores make sure every CTA of the cluster
    // has started (and finished the previous sub-block) by then
    if constexpr (VSPLIT > 1) cluster_arrive_relaxed();
    stage();
    if constexpr (!COMMIT) {
      cp_async_wait<0>();
      __syncthreads();
      conv_phase();
      __syncthreads();
      l2_phase();
      __syncthreads();
      if (t0 == 0) {
        pdl_wait();
        pdl_trigger();
      }
      gates_phase();
      __syncthreads();
    } else {
      gates_phase();
      cp_async_wait<0>();
      __syncthreads();
      conv_phase();
      __syncthreads();
      l2_phase();
      __syncthreads();
    }
    // ---- the recurrence (fused_ops.py:98-106)
    for (int t = 0; t < ntok; ++t) {
      const float decay = sm.g[t];
      const float* kt = &sm.k[t][kq * 4];
      float kr[ROWS];
      float p[4] = {0.f, 0.f, 0.f, 0.f};   // four chains: short dependent FMA sequences
#pragma unroll
      for (int i = 0; i < ROWS; i += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(kt + (i / 4) * 4 * KSPLIT);
        kr[i] = k4.x; kr[i + 1] = k4.y; kr[i + 2] = k4.z; kr[i + 3] = k4.w;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          st[i + e] *= decay;
          p[e] = fmaf(st[i + e], kr[i + e], p[e]);
        }
      }
      float pred = (p[0] + p[1]) + (p[2] + p[3]);
#pragma unroll
      for (int sh = 1; sh < KSPLIT; sh <<= 1) pred += __shfl_xor_sync(0xffffffffu, pred, sh);
      const float delta = (sm.v[t][col] - pred) * sm.beta[t];
      if (COMMIT) {
#pragma unroll
        for (int i = 0; i < ROWS; ++i) st[i] = fmaf(kr[i], delta, st[i]);
      } else {
        const float* qt = &sm.q[t][kq * 4];
        float oo[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < ROWS; i += 4) {
          const float4 q4 = *reinterpret_cast<const float4*>(qt + (i / 4) * 4 * KSPLIT);
          const float qr[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            st[i + e] = fmaf(kr[i + e], delta, st[i + e]);
            oo[e] = fmaf(st[i + e], qr[e], oo[e]);
          }
        }
        // the output sum over the KSPLIT threads is not on the state's critical path:
        // partials go to shared memory and are reduced after the loop
        sm.opart[t][col][kq] = (oo[0] + oo[1]) + (oo[2] + oo[3]);
      }
    }
    if constexpr (!COMMIT) {
      __syncthreads();
      for (int i = tid; i < ntok * COLS; i += THREADS) {
        const int t = i / COLS, c = i % COLS;
        float o = 0.f;
#pragma unroll
        for (int q = 0; q < KSPLIT; ++q) o += sm.opart[t][c][q];
        sm.o[t][c] = rbf(o);   // core tensor in the activation dtype
      }
      __syncthreads();
      // ---- gated RMSNorm over the head's Dv columns (fused/model.py:219-225).  Each CTA
      // stores its per-token sums of squares into row `rank` of every cluster CTA's
      // table, so after one cluster barrier all reads are local (and no CTA touches
      // another's shared memory once it may exit); the rows are added in rank order.
      // (Every peer is running: they all passed the cluster barrier of the conv phase and
      // wait at the one below before they go on.)
      for (int t = tid / 32; t < ntok; t += THREADS / 32) {
        float ss = 0.f;
        for (int c = tid % 32; c < COLS; c += 32) ss += sm.o[t][c] * sm.o[t][c];
        ss = warp_sum(ss);
        if (tid % 32 == 0) {
          if constexpr (VSPLIT > 1) {
            cg::cluster_group cluster = cg::this_cluster();
#pragma unroll
            for (int r = 0; r < VSPLIT; ++r) cluster.map_shared_rank(&sm.sumsq[rank][t], r)[0] = ss;
          } else {
            sm.sumsq[0][t] = ss;
          }
        }
      }
      if constexpr (VSPLIT > 1) cg::this_cluster().sync();
      else __syncthreads();
      for (int t = tid; t < ntok; t += THREADS) {
        float tot = 0.f;
        for (int r = 0; r < VSPLIT; ++r) tot += sm.sumsq[r][t];
        sm.total[t] = tot;
      }
      __syncthreads();
      for (int i = tid; i < ntok * COLS; i += THREADS) {
        const int t = i / COLS, c = i % COLS;
        const int64_t row = static_cast<int64_t>(b) * d.seq + t0 + t;
        const int vc = h * DV + vcol0 + c;
        const float inv = rsqrtf(sm.total[t] / DV + d.eps);
        const float n = rbf(sm.o[t][c] * inv);
        const float y = rbf(n * norm_w);   // c == tid % COLS for every i of this thread
        const float z = __bfloat162float(sm.zin[t][c]);
        L.out[row * vw + vc] = __float2bfloat16_rn(y * rbf(silu_f(z)));
      }
    }
    __syncthreads();   // the sub-block's shared buffers are free for the next one
  }
  if constexpr (COMMIT) {
#pragma unroll
    for (int i = 0; i < ROWS; i += 4)
      *reinterpret_cast<float4*>(scol + i) = make_float4(st[i], st[i + 1], st[i + 2], st[i + 3]);
  }
}

// New conv history after r accepted tokens: padded[r : r + K-1] (fused_ops.py:44-47).
// One thread per (layer, sequence, channel); each channel is owned by one thread, so the
// update is in place.
__global__ void gdn_conv_commit_kernel(GdnDims d, const GdnLayer* __restrict__ layers, int nlayers) {
  pdl_wait();   // the state commit (predecessor) still reads the conv tails
  pdl_trigger();
  const int64_t total = static_cast<int64_t>(nlayers) * d.batch * d.channels;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % d.channels);
    const int b = static_cast<int>((idx / d.channels) % d.batch);
    const int l = static_cast<int>(idx / (static_cast<int64_t>(d.channels) * d.batch));
    const GdnLayer& L = layers[l];
    const int r = d.accepted[b];
    if (r <= 0) continue;
    const int K1 = d.conv_k - 1;
    __nv_bfloat16* hist = L.conv_hist + (static_cast<int64_t>(d.slots[b]) * d.channels + c) * K1;
    __nv_bfloat16 nh[QW_MAX_CONV];
    for (int j = 0; j < K1; ++j) {
      const int p = r + j;  // index into padded = [hist(K-1) | proj(seq)]
      nh[j] = p < K1 ? hist[p] : L.proj[(static_cast<int64_t>(b) * d.seq + (p - K1)) * d.ldp + c];
    }
    for (int j = 0; j < K1; ++j) hist[j] = nh[j];
  }
}

template <int DK, int DV, int VSPLIT, bool COMMIT>
static int launch_block(const GdnDims& d, const GdnLayer* layers, int layer0, int nlayers,
                        cudaStream_t s) {
  using Tile = GdnTile<DK, DV, VSPLIT>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(VSPLIT, d.v_heads, d.batch * nlayers);
  cfg.blockDim = dim3(Tile::THREADS);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = VSPLIT;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gdn_block_kernel<DK, DV, VSPLIT, COMMIT>, d, layers, layer0);
  if (e != cudaSuccess) return cuda_status(e, COMMIT ? "gdn_commit" : "gdn_verify");
  return QW_OK;
}

template <bool COMMIT>
static int dispatch_block(const GdnDims& d, const GdnLayer* layers, int layer0, int nlayers,
                          cudaStream_t s) {
  if (d.dk == 128 && d.dv == 128) return launch_block<128, 128, 4, COMMIT>(d, layers, layer0, nlayers, s);
  if (d.dk == 64 && d.dv == 64) return launch_block<64, 64, 2, COMMIT>(d, layers, layer0, nlayers, s);
  if (d.dk == 128 && d.dv == 64) return launch_block<128, 64, 2, COMMIT>(d, layers, layer0, nlayers, s);
  return fail(QW_ERR_UNSUPPORTED, "gdn block: head dims (%d,%d) not built", d.dk, d.dv);
}

static int check_dims(const GdnDims& d) {
  QW_CHECK_ARG(d.batch >= 1 && d.seq >= 1 && d.seq <= QW_MAX_SEQ,
               "gdn block: need 1 <= seq <= %d", QW_MAX_SEQ);
  QW_CHECK_ARG(d.v_heads >= 1 && d.k_heads >= 1 && d.v_heads % d.k_heads == 0,
               "gdn block: value heads must be a multiple of key heads");
  QW_CHECK_ARG(d.conv_k >= 2 && d.conv_k <= QW_MAX_CONV, "gdn block: conv kernel out of range");
  if (d.conv_k != GDN_CONV_K)
    return fail(QW_ERR_UNSUPPORTED, "gdn block: conv kernel width %d not built (%d)", d.conv_k, GDN_CONV_K);
  QW_CHECK_ARG(d.channels == 2 * d.k_heads * d.dk + d.v_heads * d.dv, "gdn block: channel count");
  QW_CHECK_ARG(d.ldp >= d.channels + d.v_heads * d.dv, "gdn block: projection row too short");
  QW_CHECK_ARG(d.ldp % 8 == 0, "gdn block: the projection row stride must be a multiple of 8 elements");
  QW_CHECK_ARG(d.slots != nullptr, "gdn block: null slot table");
  return QW_OK;
}

}  // namespace qw

using namespace qw;

extern "C" int qw_gated_delta_rule(const void* q, const void* k, const void* v, const void* g,
                                   const void* beta, int in_dtype, const void* state0,
                                   int state_dtype, const int16_t* eff_len, void* core,
                                   void* state_out, int64_t batch, int64_t seq, int64_t heads,
                                   int64_t dk, int64_t dv, int use_l2norm, void* stream) {
  QW_CHECK_ARG(q && k && v && g && beta && state0 && eff_len && core && state_out,
               "chunk_gated_delta_rule: null pointer");
  QW_CHECK_ARG(batch >= 1 && seq >= 1 && heads >= 1 && dk >= 1 && dv >= 1,
               "GDN requires compatible [B,S,H,D] tensors and [B,S,H] gates");
  QW_CHECK_ARG(dk <= 256 && dv <= 256 && dk * dv <= 48 * 1024, "chunk_gated_delta_rule: head too large");
  QW_CHECK_ARG(batch < 65536 && heads < 65536, "chunk_gated_delta_rule: grid too large");
  const size_t smem = (static_cast<size_t>(dk) * dv + 2 * dk + 64) * sizeof(float);
  cudaStream_t s = as_stream(stream);
  dim3 grid(static_cast<unsigned>(heads), static_cast<unsigned>(batch));
  const int threads = 128;
#define QW_GDN(TIN, TST)                                                                       \
  do {                                                                                         \
    auto kern = gdn_rule_kernel<TIN, TST>;                                                     \
    if (smem > 48 * 1024) {                                                                    \
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                                           static_cast<int>(smem));                            \
      if (e != cudaSuccess) return cuda_status(e, "chunk_gated_delta_rule smem");              \
    }                                                                                          \
    kern<<<grid, threads, smem, s>>>(                                                          \
        static_cast<const TIN*>(q), static_cast<const TIN*>(k), static_cast<const TIN*>(v),    \
        static_cast<const TIN*>(g), static_cast<const TIN*>(beta),                             \
        static_cast<const TST*>(state0), eff_len, static_cast<TIN*>(core),                     \
        static_cast<TST*>(state_out), static_cast<int>(seq), static_cast<int>(heads),          \
        static_cast<int>(dk), static_cast<int>(dv), use_l2norm);                               \
  } while (0)
  if (state_dtype == QW_F32) {
    switch (in_dtype) {
      case QW_F32: QW_GDN(float, float); break;
      case QW_F16: QW_GDN(__half, float); break;
      case QW_BF16: QW_GDN(__nv_bfloat16, float); break;
      default: return fail(QW_ERR_ARG, "chunk_gated_delta_rule: bad input dtype");
    }
  } else if (state_dtype == QW_F16) {
    switch (in_dtype) {
      case QW_F32: QW_GDN(float, __half); break;
      case QW_F16: QW_GDN(__half, __half); break;
      case QW_BF16: QW_GDN(__nv_bfloat16, __half); break;
      default: return fail(QW_ERR_ARG, "chunk_gated_delta_rule: bad input dtype");
    }
  } else {
    return fail(QW_ERR_ARG, "initial_state must be FP16/FP32 [B,H,Dk,Dv]");
  }
#undef QW_GDN
  QW_LAUNCH_CHECK("chunk_gated_delta_rule");
  return QW_OK;
}

extern "C" int qw_gdn_verify(const qw_gdn_dims* dims, const qw_gdn_layer* layers_dev, int layer,
                             void* stream) {
  QW_CHECK_ARG(dims && layers_dev && layer >= 0, "gdn_verify: null argument");
  int st = check_dims(*dims);
  if (st) return st;
  return dispatch_block<false>(*dims, layers_dev, layer, 1, as_stream(stream));
}

extern "C" int qw_gdn_commit(const qw_gdn_dims* dims, const qw_gdn_layer* layers_dev, int nlayers,
                             void* stream) {
  QW_CHECK_ARG(dims && layers_dev && nlayers >= 1, "gdn_commit: null argument");
  int st = check_dims(*dims);
  if (st) return st;
  QW_CHECK_ARG(dims->accepted != nullptr, "gdn_commit: null accepted counts");
  cudaStream_t s = as_stream(stream);
  st = dispatch_block<true>(*dims, layers_dev, 0, nlayers, s);
  if (st) return st;
  const int64_t total = static_cast<int64_t>(nlayers) * dims->batch * dims->channels;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  QW_LAUNCH_PDL("gdn_conv_commit", gdn_conv_commit_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s,
                *dims, layers_dev, nlayers);
  return QW_OK;
}
