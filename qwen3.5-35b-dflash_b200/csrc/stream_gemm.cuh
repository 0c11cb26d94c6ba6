// Weight-streaming skinny GEMM core shared by the linear, MoE and lm_head kernels.
//
// y[t, n] = sum_k x[t, k] * W[n, k] for a handful of tokens t (a verify block) and a
// weight matrix streamed once from HBM.  The weight is the tensor-core A operand
// (16 output rows per warp tile), the tokens are the B operand (8 per n-tile).  Nothing
// is staged in shared memory: every lane loads its own fragments from global memory
// with 16-byte loads, so each warp issues all of its loads at once and runs without a
// CTA barrier until the cross-warp K reduction.
//
// K permutation.  The dot product is invariant under any permutation of k applied to
// both operands.  Within every 32-wide block of K the weight streams are packed in the
// order that makes lane (gid, tig)'s B fragments of two consecutive k16-steps the 8
// contiguous activations x[t, 32p + 8*tig .. +7]: mma-logical k = 16*(2p+h) + 2*tig + e
// (+8 for the second register) is physical k = 32p + 8*tig + 4h + e (+2).
//
//   W4 stream (int4 symmetric, bf16 scale per G-wide K group), per 16-row tile and per
//   group a chunk of 8*G + 32 bytes: G/16 k16-steps x 32 lanes x one 32-bit word (eight
//   offset-binary nibbles, see dequant_w4_word), grouped in 16-byte vectors
//   [vector v][lane][min(4, G/16) words], then the 16 bf16 scales ordered
//   (row 0, row 8, row 1, row 9, ...) so that lane (gid) reads its pair as one word.
//   Scales are applied in fp32 to the per-group partial sums, so the product equals
//   x . (q * scale) up to fp32 summation order.
//
//   B16 stream (bf16), per 16-row tile and 64-wide K chunk 2048 bytes: 4 k16-steps x
//   32 lanes x one 16-byte vector holding the lane's 4 A-fragment registers.
//
//   Row format: a plain row-major [N, K] 16-bit matrix (the fused-ops ABI passes dense
//   expert weights); fragments use the natural k order and 32-bit loads.
#pragma once

#include "qw_common.cuh"

namespace qw {

constexpr int SG_WARPS = 8;

// OT_ is the tensor-core operand type: bf16 (the activations as stored), or fp16 (exact
// for the int4 weights and for bf16 activations in [2^-14, 65504]; the decode then needs
// no conversion-unit work, but the activations are converted as they are loaded).
template <int G, typename OT_ = __nv_bfloat16>
struct W4Fmt {
  using ET = __nv_bfloat16;   // activation storage
  using OT = OT_;
  static constexpr int KCHUNK = G;
  static constexpr int STEPS = G / 16;
  static constexpr int WORDS = STEPS;              // 32-bit words per lane per chunk
  static constexpr int VW = STEPS < 4 ? STEPS : 4; // words per vector load
  static constexpr int NV = STEPS / VW;
  static constexpr int CHB = 8 * G + 32;
  static constexpr bool SCALED = true;
  static constexpr bool PERMUTED_K = true;
  static constexpr bool NIB = false;

  __host__ __device__ static int64_t tile_offset(int64_t rt, int k, int64_t /*ld*/) {
    return rt * (k / G) * static_cast<int64_t>(CHB);
  }
  __device__ __forceinline__ static void load(const uint8_t* tile, int c, int lane, int64_t /*ld*/,
                                              uint32_t (&w)[WORDS], uint32_t& sc) {
    const uint8_t* chunk = tile + static_cast<int64_t>(c) * CHB;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const uint8_t* p = chunk + v * (32 * VW * 4) + lane * (VW * 4);
      if constexpr (VW == 4) {
        uint4 u = ldg_stream(p);
        w[v * 4 + 0] = u.x; w[v * 4 + 1] = u.y; w[v * 4 + 2] = u.z; w[v * 4 + 3] = u.w;
      } else {
        uint2 u = ldg_stream2(p);
        w[v * 2 + 0] = u.x; w[v * 2 + 1] = u.y;
      }
    }
    sc = __ldg(reinterpret_cast<const uint32_t*>(chunk + 8 * G + (lane >> 2) * 4));
  }
  __device__ __forceinline__ static void afrag(const uint32_t (&w)[WORDS], int s, uint32_t (&a)[4]) {
    if constexpr (std::is_same<OT, __half>::value) dequant_w4_word_f16(w[s], a);
    else dequant_w4_word(w[s], a);
  }
};

// W4 chunks entering the MMA as raw nibbles (w4_nibbles_f16), the offset restored per
// chunk from the activation sums exactly as w4n_smem_chunk / w4n_smem_pair compute it, so
// the streaming and the shared-memory kernels give a token the same bits.
template <int G>
struct W4NibFmt : W4Fmt<G, __half> {
  static constexpr bool NIB = true;
  __device__ __forceinline__ static void afrag(const uint32_t (&w)[G / 16], int s, uint32_t (&a)[4]) {
    w4_nibbles_f16(w[s], a);
  }
};

struct B16Fmt {
  using ET = __nv_bfloat16;
  using OT = __nv_bfloat16;
  static constexpr int KCHUNK = 64;
  static constexpr int STEPS = 4;
  static constexpr int WORDS = 16;
  static constexpr int CHB = 2048;
  static constexpr bool SCALED = false;
  static constexpr bool PERMUTED_K = true;
  static constexpr bool NIB = false;

  __host__ __device__ static int64_t tile_offset(int64_t rt, int k, int64_t /*ld*/) {
    return rt * (k / 64) * static_cast<int64_t>(CHB);
  }
  __device__ __forceinline__ static void load(const uint8_t* tile, int c, int lane, int64_t /*ld*/,
                                              uint32_t (&w)[WORDS], uint32_t& sc) {
    const uint8_t* chunk = tile + static_cast<int64_t>(c) * CHB;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      uint4 u = ldg_stream(chunk + s * 512 + lane * 16);
      w[s * 4 + 0] = u.x; w[s * 4 + 1] = u.y; w[s * 4 + 2] = u.z; w[s * 4 + 3] = u.w;
    }
    sc = 0;
  }
  __device__ __forceinline__ static void afrag(const uint32_t (&w)[WORDS], int s, uint32_t (&a)[4]) {
    a[0] = w[s * 4 + 0]; a[1] = w[s * 4 + 1]; a[2] = w[s * 4 + 2]; a[3] = w[s * 4 + 3];
  }
};

// Row-major 16-bit matrix [N, K] with row stride `ld` bytes; natural k order.
template <typename ET_>
struct RowFmt {
  using ET = ET_;
  using OT = ET_;
  static constexpr int KCHUNK = 32;
  static constexpr int STEPS = 2;
  static constexpr int WORDS = 8;
  static constexpr bool SCALED = false;
  static constexpr bool PERMUTED_K = false;
  static constexpr bool NIB = false;

  __host__ __device__ static int64_t tile_offset(int64_t rt, int /*k*/, int64_t ld) {
    return rt * 16 * ld;
  }
  __device__ __forceinline__ static void load(const uint8_t* tile, int c, int lane, int64_t ld,
                                              uint32_t (&w)[WORDS], uint32_t& sc) {
    const int gid = lane >> 2, tig = lane & 3;
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const uint8_t* p = tile + static_cast<int64_t>(gid) * ld + (c * 32 + s * 16 + 2 * tig) * 2;
      w[s * 4 + 0] = __ldg(reinterpret_cast<const uint32_t*>(p));
      w[s * 4 + 1] = __ldg(reinterpret_cast<const uint32_t*>(p + 8 * ld));
      w[s * 4 + 2] = __ldg(reinterpret_cast<const uint32_t*>(p + 16));
      w[s * 4 + 3] = __ldg(reinterpret_cast<const uint32_t*>(p + 8 * ld + 16));
    }
    sc = 0;
  }
  __device__ __forceinline__ static void afrag(const uint32_t (&w)[WORDS], int s, uint32_t (&a)[4]) {
    a[0] = w[s * 4 + 0]; a[1] = w[s * 4 + 1]; a[2] = w[s * 4 + 2]; a[3] = w[s * 4 + 3];
  }
};

// Sum of 8 packed fp16 values in fp32, in order.
__device__ __forceinline__ float sum8_f16(uint4 v) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[e]));
    s += f.x;
    s += f.y;
  }
  return s;
}

// Sum X of one token's G fp16 activations of one K group, in fp32 and in a fixed order
// that the lanes of an MMA fragment group (and a warp converting the activations)
// reproduce: p(q, t) = the 8 values at k = 32q + 8t .. +7 summed in order, S_t = p(0, t)
// + p(1, t) + ... in order of q, X = (S0 + S1) + (S2 + S3).  p: 16-byte aligned.
template <int G>
__device__ __forceinline__ float group_xsum_f16(const __half* p) {
  float s[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    s[t] = sum8_f16(*reinterpret_cast<const uint4*>(p + 8 * t));
#pragma unroll
    for (int q = 1; q < G / 32; ++q) s[t] += sum8_f16(*reinterpret_cast<const uint4*>(p + 32 * q + 8 * t));
  }
  return (s[0] + s[1]) + (s[2] + s[3]);
}

// The same sum from a warp whose lane l holds the 8 values of segment l (k = 8l .. 8l+7
// of 256 consecutive activations of one token, i.e. 256 / G whole groups): returns X of
// the lane's group on the lanes holding a group's first segment.  All lanes call it.
template <int G>
__device__ __forceinline__ float warp_group_xsum_f16(float p, int lane) {
  float s = p;
#pragma unroll
  for (int q = 1; q < G / 32; ++q) s += __shfl_down_sync(0xffffffffu, p, 4 * q);
  const float a = s + __shfl_xor_sync(0xffffffffu, s, 1);
  return a + __shfl_xor_sync(0xffffffffu, a, 2);
}

// Activation rows of the lane's n-tiles: n-tile j covers tokens j*8 .. j*8+7, the lane
// reads token j*8 + gid.  Rows are element pointers to x[token, 0].
template <typename ET, int NT>
struct XRows {
  const ET* r[NT];
};

// Weight fragments of one chunk, and the activation fragments of one chunk.
template <class Fmt>
struct WFrag {
  uint32_t w[Fmt::WORDS];
  uint32_t sc;
};
template <class Fmt, int NT>
struct BFrag {
  uint32_t b[Fmt::KCHUNK / 32][NT][4];
};

template <class Fmt>
__device__ __forceinline__ void load_w(WFrag<Fmt>& f, const uint8_t* tile, int c, int lane, int64_t ld) {
  Fmt::load(tile, c, lane, ld, f.w, f.sc);
}

template <class Fmt, int NT>
__device__ __forceinline__ void load_b(BFrag<Fmt, NT>& f, int c, int lane, const XRows<typename Fmt::ET, NT>& x) {
  const int kb = c * Fmt::KCHUNK;
  const int tig = lane & 3;
#pragma unroll
  for (int q = 0; q < Fmt::KCHUNK / 32; ++q) {
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      if constexpr (Fmt::PERMUTED_K) {
        uint4 v = __ldg(reinterpret_cast<const uint4*>(x.r[j] + kb + 32 * q + 8 * tig));
        if constexpr (!std::is_same<typename Fmt::ET, typename Fmt::OT>::value) v = bf16x8_to_f16x8(v);
        f.b[q][j][0] = v.x; f.b[q][j][1] = v.y; f.b[q][j][2] = v.z; f.b[q][j][3] = v.w;
      } else {
        const typename Fmt::ET* p = x.r[j] + kb + 32 * q + 2 * tig;
        f.b[q][j][0] = __ldg(reinterpret_cast<const uint32_t*>(p));
        f.b[q][j][1] = __ldg(reinterpret_cast<const uint32_t*>(p + 8));
        f.b[q][j][2] = __ldg(reinterpret_cast<const uint32_t*>(p + 16));
        f.b[q][j][3] = __ldg(reinterpret_cast<const uint32_t*>(p + 24));
      }
    }
  }
}

template <class Fmt, int NT>
__device__ __forceinline__ void mma_frag(const WFrag<Fmt>& wf, const BFrag<Fmt, NT>& bf, float (&acc)[NT][4]) {
  using ET = typename Fmt::OT;
  if constexpr (Fmt::NIB) {
    float part[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) part[j][0] = part[j][1] = part[j][2] = part[j][3] = 0.f;
#pragma unroll
    for (int s = 0; s < Fmt::STEPS; ++s) {
      uint32_t a[4];
      Fmt::afrag(wf.w, s, a);
#pragma unroll
      for (int j = 0; j < NT; ++j)
        mma_f16_16816(part[j], a, bf.b[s >> 1][j][(s & 1) * 2], bf.b[s >> 1][j][(s & 1) * 2 + 1]);
    }
    // the chunk's activation sums in group_xsum_f16's order: this lane's running sum
    // over its 8-value segments, then the fragment group's four lanes combined, then
    // moved to the lanes holding each accumulator column
    const int tig = threadIdx.x & 3;
    const float2 s2 = bf162_to_f2(wf.sc);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      float sx = sum8_f16(make_uint4(bf.b[0][j][0], bf.b[0][j][1], bf.b[0][j][2], bf.b[0][j][3]));
#pragma unroll
      for (int q = 1; q < Fmt::KCHUNK / 32; ++q)
        sx += sum8_f16(make_uint4(bf.b[q][j][0], bf.b[q][j][1], bf.b[q][j][2], bf.b[q][j][3]));
      const float pa = sx + __shfl_xor_sync(0xffffffffu, sx, 1);
      const float xg = pa + __shfl_xor_sync(0xffffffffu, pa, 2);
      const float x0 = -8.f * __shfl_sync(0xffffffffu, xg, 8 * tig);
      const float x1 = -8.f * __shfl_sync(0xffffffffu, xg, 8 * tig + 4);
      acc[j][0] = fmaf(fmaf(part[j][0], 0x1p24f, x0), s2.x, acc[j][0]);
      acc[j][1] = fmaf(fmaf(part[j][1], 0x1p24f, x1), s2.x, acc[j][1]);
      acc[j][2] = fmaf(fmaf(part[j][2], 0x1p20f, x0), s2.y, acc[j][2]);
      acc[j][3] = fmaf(fmaf(part[j][3], 0x1p20f, x1), s2.y, acc[j][3]);
    }
  } else if constexpr (Fmt::SCALED) {
    float part[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) part[j][0] = part[j][1] = part[j][2] = part[j][3] = 0.f;
#pragma unroll
    for (int s = 0; s < Fmt::STEPS; ++s) {
      uint32_t a[4];
      Fmt::afrag(wf.w, s, a);
#pragma unroll
      for (int j = 0; j < NT; ++j)
        mma16816<ET>(part[j], a, bf.b[s >> 1][j][(s & 1) * 2], bf.b[s >> 1][j][(s & 1) * 2 + 1]);
    }
    const float2 s2 = bf162_to_f2(wf.sc);  // (row gid, row gid + 8)
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      acc[j][0] = fmaf(part[j][0], s2.x, acc[j][0]);
      acc[j][1] = fmaf(part[j][1], s2.x, acc[j][1]);
      acc[j][2] = fmaf(part[j][2], s2.y, acc[j][2]);
      acc[j][3] = fmaf(part[j][3], s2.y, acc[j][3]);
    }
  } else {
#pragma unroll
    for (int s = 0; s < Fmt::STEPS; ++s) {
      uint32_t a[4];
      Fmt::afrag(wf.w, s, a);
#pragma unroll
      for (int j = 0; j < NT; ++j)
        mma16816<ET>(acc[j], a, bf.b[s >> 1][j][(s & 1) * 2], bf.b[s >> 1][j][(s & 1) * 2 + 1]);
    }
  }
}

// Stream chunks [c0, c1) of NTILES row tiles that share the activations: the weights
// run PF chunks ahead in a register ring (issued first, before anything else, so the
// HBM latency overlaps the caller's setup), the activations (L1/L2 hits) one chunk
// ahead.  PF must be even.
// With PDL the first weight chunks are requested before pdl_wait(): weights are never
// written by a kernel, the activations come from the predecessor.
template <class Fmt, int NT, int PF, int NTILES, bool PDL = false>
__device__ __forceinline__ void stream_tiles(const uint8_t* const (&tiles)[NTILES], int64_t ld, int c0, int c1,
                                             int lane, const XRows<typename Fmt::ET, NT>& x,
                                             float (&acc)[NTILES][NT][4]) {
  static_assert(PF % 2 == 0, "PF must be even");
  WFrag<Fmt> w[PF][NTILES];
  BFrag<Fmt, NT> b[2];
#pragma unroll
  for (int p = 0; p < PF; ++p)
    if (c0 + p < c1) {
#pragma unroll
      for (int t = 0; t < NTILES; ++t) load_w<Fmt>(w[p][t], tiles[t], c0 + p, lane, ld);
    }
  if constexpr (PDL) {
    pdl_wait();
    pdl_trigger();
  }
  if (c0 < c1) load_b<Fmt, NT>(b[0], c0, lane, x);
  for (int c = c0; c < c1; c += PF) {
#pragma unroll
    for (int p = 0; p < PF; ++p) {
      if (c + p < c1) {
        if (c + p + 1 < c1) load_b<Fmt, NT>(b[(p + 1) & 1], c + p + 1, lane, x);
#pragma unroll
        for (int t = 0; t < NTILES; ++t) mma_frag<Fmt, NT>(w[p][t], b[p & 1], acc[t]);
        if (c + p + PF < c1) {
#pragma unroll
          for (int t = 0; t < NTILES; ++t) load_w<Fmt>(w[p][t], tiles[t], c + p + PF, lane, ld);
        }
      }
    }
  }
}

template <class Fmt, int NT, int PF, bool PDL = false>
__device__ __forceinline__ void stream_tile(const uint8_t* tile, int64_t ld, int c0, int c1, int lane,
                                            const XRows<typename Fmt::ET, NT>& x, float (&acc)[NT][4]) {
  const uint8_t* const tiles[1] = {tile};
  float (&a1)[1][NT][4] = *reinterpret_cast<float (*)[1][NT][4]>(&acc);
  stream_tiles<Fmt, NT, PF, 1, PDL>(tiles, ld, c0, c1, lane, x, a1);
}

// acc[nt] += W4 chunk (16 rows x G, shared memory) . x rows, the weights entering the MMA
// as their raw nibbles (w4_nibbles_f16: no decode arithmetic) and the offset and nibble
// position restored per chunk: d = 2^24 P - 8 X (rows gid) or 2^20 P - 8 X (rows gid + 8),
// acc += d * scale.  xq[nt][e]: the chunk sums (group_xsum_f16) of the token of
// accumulator column 2 tig + e of n-tile nt, indexed by the global chunk cg.
template <int G, int NT>
__device__ __forceinline__ void w4n_smem_chunk(const uint8_t* chunk, const __half* const (&xr)[2], int k0,
                                               const float* const (&xq)[2][2], int cg, int lane,
                                               float (&acc)[2][4]) {
  using Fmt = W4Fmt<G>;
  uint32_t w[Fmt::WORDS];
#pragma unroll
  for (int v = 0; v < Fmt::NV; ++v) {
    const uint8_t* p = chunk + v * (32 * Fmt::VW * 4) + lane * (Fmt::VW * 4);
    if constexpr (Fmt::VW == 4) {
      const uint4 u = *reinterpret_cast<const uint4*>(p);
      w[v * 4 + 0] = u.x; w[v * 4 + 1] = u.y; w[v * 4 + 2] = u.z; w[v * 4 + 3] = u.w;
    } else {
      const uint2 u = *reinterpret_cast<const uint2*>(p);
      w[v * 2 + 0] = u.x; w[v * 2 + 1] = u.y;
    }
  }
  const uint32_t sc = *reinterpret_cast<const uint32_t*>(chunk + 8 * G + (lane >> 2) * 4);
  const int tig = lane & 3;
  float part[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) part[j][0] = part[j][1] = part[j][2] = part[j][3] = 0.f;
#pragma unroll
  for (int q = 0; q < G / 32; ++q) {
    uint32_t b[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr[j] + k0 + 32 * q + 8 * tig);
      b[j][0] = v.x; b[j][1] = v.y; b[j][2] = v.z; b[j][3] = v.w;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t a[4];
      w4_nibbles_f16(w[2 * q + h], a);
#pragma unroll
      for (int j = 0; j < NT; ++j) mma_f16_16816(part[j], a, b[j][2 * h], b[j][2 * h + 1]);
    }
  }
  const float2 s2 = bf162_to_f2(sc);
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const float x0 = -8.f * xq[j][0][cg], x1 = -8.f * xq[j][1][cg];
    acc[j][0] = fmaf(fmaf(part[j][0], 0x1p24f, x0), s2.x, acc[j][0]);
    acc[j][1] = fmaf(fmaf(part[j][1], 0x1p24f, x1), s2.x, acc[j][1]);
    acc[j][2] = fmaf(fmaf(part[j][2], 0x1p20f, x0), s2.y, acc[j][2]);
    acc[j][3] = fmaf(fmaf(part[j][3], 0x1p20f, x1), s2.y, acc[j][3]);
  }
}

// The same for two tiles over the same k range at once (an expert's gate and up rows):
// one x fragment load feeds two independent MMA chains.  Per tile the MMA sequence and
// the epilogue are those of w4n_smem_chunk, so each result has the same bits.  One
// n-tile: xr the lane's B-fragment token row, xq0 / xq1 the chunk sums of the tokens of
// accumulator columns 2 tig, 2 tig + 1.
template <int G>
__device__ __forceinline__ void w4n_smem_pair(const uint8_t* ca, const uint8_t* cb, const __half* xr, int k0,
                                              const float* xq0, const float* xq1, int cg, int lane,
                                              float (&acca)[4], float (&accb)[4]) {
  using Fmt = W4Fmt<G>;
  uint32_t wa[Fmt::WORDS], wb[Fmt::WORDS];
#pragma unroll
  for (int v = 0; v < Fmt::NV; ++v) {
    const int off = v * (32 * Fmt::VW * 4) + lane * (Fmt::VW * 4);
    if constexpr (Fmt::VW == 4) {
      const uint4 u = *reinterpret_cast<const uint4*>(ca + off);
      const uint4 t = *reinterpret_cast<const uint4*>(cb + off);
      wa[v * 4 + 0] = u.x; wa[v * 4 + 1] = u.y; wa[v * 4 + 2] = u.z; wa[v * 4 + 3] = u.w;
      wb[v * 4 + 0] = t.x; wb[v * 4 + 1] = t.y; wb[v * 4 + 2] = t.z; wb[v * 4 + 3] = t.w;
    } else {
      const uint2 u = *reinterpret_cast<const uint2*>(ca + off);
      const uint2 t = *reinterpret_cast<const uint2*>(cb + off);
      wa[v * 2 + 0] = u.x; wa[v * 2 + 1] = u.y;
      wb[v * 2 + 0] = t.x; wb[v * 2 + 1] = t.y;
    }
  }
  const uint32_t sca = *reinterpret_cast<const uint32_t*>(ca + 8 * G + (lane >> 2) * 4);
  const uint32_t scb = *reinterpret_cast<const uint32_t*>(cb + 8 * G + (lane >> 2) * 4);
  const int tig = lane & 3;
  float pa[4] = {0.f, 0.f, 0.f, 0.f}, pb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int q = 0; q < G / 32; ++q) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + k0 + 32 * q + 8 * tig);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t b0 = h ? v.z : v.x, b1 = h ? v.w : v.y;
      uint32_t a[4];
      w4_nibbles_f16(wa[2 * q + h], a);
      mma_f16_16816(pa, a, b0, b1);
      w4_nibbles_f16(wb[2 * q + h], a);
      mma_f16_16816(pb, a, b0, b1);
    }
  }
  const float x0 = -8.f * xq0[cg], x1 = -8.f * xq1[cg];
  const float2 s2a = bf162_to_f2(sca), s2b = bf162_to_f2(scb);
  acca[0] = fmaf(fmaf(pa[0], 0x1p24f, x0), s2a.x, acca[0]);
  acca[1] = fmaf(fmaf(pa[1], 0x1p24f, x1), s2a.x, acca[1]);
  acca[2] = fmaf(fmaf(pa[2], 0x1p20f, x0), s2a.y, acca[2]);
  acca[3] = fmaf(fmaf(pa[3], 0x1p20f, x1), s2a.y, acca[3]);
  accb[0] = fmaf(fmaf(pb[0], 0x1p24f, x0), s2b.x, accb[0]);
  accb[1] = fmaf(fmaf(pb[1], 0x1p24f, x1), s2b.x, accb[1]);
  accb[2] = fmaf(fmaf(pb[2], 0x1p20f, x0), s2b.y, accb[2]);
  accb[3] = fmaf(fmaf(pb[3], 0x1p20f, x1), s2b.y, accb[3]);
}

// NC consecutive chunk pairs (chunks cg .. cg + NC - 1 of both tiles, CHB apart) at once:
// 2 NC independent MMA chains in flight.  Each chunk's MMA sequence and its epilogue, in
// chunk order, are those of NC calls of w4n_smem_pair, so the results have the same bits.
template <int G, int NC>
__device__ __forceinline__ void w4n_smem_pairs(const uint8_t* ca, const uint8_t* cb, const __half* xr, int k0,
                                               const float* xq0, const float* xq1, int cg, int lane,
                                               float (&acca)[4], float (&accb)[4]) {
  using Fmt = W4Fmt<G>;
  uint32_t wa[NC][Fmt::WORDS], wb[NC][Fmt::WORDS];
  uint32_t sca[NC], scb[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
#pragma unroll
    for (int v = 0; v < Fmt::NV; ++v) {
      const int off = c * Fmt::CHB + v * (32 * Fmt::VW * 4) + lane * (Fmt::VW * 4);
      if constexpr (Fmt::VW == 4) {
        const uint4 u = *reinterpret_cast<const uint4*>(ca + off);
        const uint4 t = *reinterpret_cast<const uint4*>(cb + off);
        wa[c][v * 4 + 0] = u.x; wa[c][v * 4 + 1] = u.y; wa[c][v * 4 + 2] = u.z; wa[c][v * 4 + 3] = u.w;
        wb[c][v * 4 + 0] = t.x; wb[c][v * 4 + 1] = t.y; wb[c][v * 4 + 2] = t.z; wb[c][v * 4 + 3] = t.w;
      } else {
        const uint2 u = *reinterpret_cast<const uint2*>(ca + off);
        const uint2 t = *reinterpret_cast<const uint2*>(cb + off);
        wa[c][v * 2 + 0] = u.x; wa[c][v * 2 + 1] = u.y;
        wb[c][v * 2 + 0] = t.x; wb[c][v * 2 + 1] = t.y;
      }
    }
    sca[c] = *reinterpret_cast<const uint32_t*>(ca + c * Fmt::CHB + 8 * G + (lane >> 2) * 4);
    scb[c] = *reinterpret_cast<const uint32_t*>(cb + c * Fmt::CHB + 8 * G + (lane >> 2) * 4);
  }
  const int tig = lane & 3;
  float pa[NC][4], pb[NC][4];
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int r = 0; r < 4; ++r) pa[c][r] = pb[c][r] = 0.f;
#pragma unroll
  for (int q = 0; q < G / 32; ++q) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + k0 + c * G + 32 * q + 8 * tig);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t b0 = h ? v.z : v.x, b1 = h ? v.w : v.y;
        uint32_t a[4];
        w4_nibbles_f16(wa[c][2 * q + h], a);
        mma_f16_16816(pa[c], a, b0, b1);
        w4_nibbles_f16(wb[c][2 * q + h], a);
        mma_f16_16816(pb[c], a, b0, b1);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const float x0 = -8.f * xq0[cg + c], x1 = -8.f * xq1[cg + c];
    const float2 s2a = bf162_to_f2(sca[c]), s2b = bf162_to_f2(scb[c]);
    acca[0] = fmaf(fmaf(pa[c][0], 0x1p24f, x0), s2a.x, acca[0]);
    acca[1] = fmaf(fmaf(pa[c][1], 0x1p24f, x1), s2a.x, acca[1]);
    acca[2] = fmaf(fmaf(pa[c][2], 0x1p20f, x0), s2a.y, acca[2]);
    acca[3] = fmaf(fmaf(pa[c][3], 0x1p20f, x1), s2a.y, acca[3]);
    accb[0] = fmaf(fmaf(pb[c][0], 0x1p24f, x0), s2b.x, accb[0]);
    accb[1] = fmaf(fmaf(pb[c][1], 0x1p24f, x1), s2b.x, accb[1]);
    accb[2] = fmaf(fmaf(pb[c][2], 0x1p20f, x0), s2b.y, accb[2]);
    accb[3] = fmaf(fmaf(pb[c][3], 0x1p20f, x1), s2b.y, accb[3]);
  }
}

// n consecutive chunks (global chunk index cg0 + c) through w4n_smem_chunk; NT = 2 only
// when the unit has > 8 tokens.
template <int G>
__device__ __forceinline__ void w4n_smem_run(const uint8_t* chunk, int n, const __half* const (&xr)[2], int k0,
                                             const float* const (&xq)[2][2], int cg0, int lane, bool two,
                                             float (&acc)[2][4]) {
  constexpr int CHB = W4Fmt<G>::CHB;
  if (two) {
    for (int c = 0; c < n; ++c) w4n_smem_chunk<G, 2>(chunk + c * CHB, xr, k0 + c * G, xq, cg0 + c, lane, acc);
  } else {
    for (int c = 0; c < n; ++c) w4n_smem_chunk<G, 1>(chunk + c * CHB, xr, k0 + c * G, xq, cg0 + c, lane, acc);
  }
}

// acc[nt] += W4 chunks c0 .. c0+NC-1 (16 rows x G each, consecutive in shared memory)
// . x rows (token of lane gid in n-tile nt at xr[nt]).  NC chunks are decoded and
// multiplied interleaved (independent instruction streams for one warp) and their
// scaled partial sums are added to acc in chunk order, as one chunk at a time would.
// Both operands are fp16: the weights are small integers and the activations are bf16
// values, exact in fp16 (|x| in [2^-14, 65504]), so the products equal the bf16 ones and
// the decode needs no conversion-unit instructions (dequant_w4_word_f16).
template <int G, int NC, int NT, typename OT = __half>
__device__ __forceinline__ void w4_smem_chunks(const uint8_t* chunk, const OT* const (&xr)[2], int k0,
                                          int lane, float (&acc)[2][4]) {
  using Fmt = W4Fmt<G>;
  uint32_t w[NC][Fmt::WORDS];
  uint32_t sc[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
#pragma unroll
    for (int v = 0; v < Fmt::NV; ++v) {
      const uint8_t* p = chunk + c * Fmt::CHB + v * (32 * Fmt::VW * 4) + lane * (Fmt::VW * 4);
      if constexpr (Fmt::VW == 4) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        w[c][v * 4 + 0] = u.x; w[c][v * 4 + 1] = u.y; w[c][v * 4 + 2] = u.z; w[c][v * 4 + 3] = u.w;
      } else {
        const uint2 u = *reinterpret_cast<const uint2*>(p);
        w[c][v * 2 + 0] = u.x; w[c][v * 2 + 1] = u.y;
      }
    }
    sc[c] = *reinterpret_cast<const uint32_t*>(chunk + c * Fmt::CHB + 8 * G + (lane >> 2) * 4);
  }
  const int tig = lane & 3;
  float part[NC][NT][4];
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int j = 0; j < NT; ++j) part[c][j][0] = part[c][j][1] = part[c][j][2] = part[c][j][3] = 0.f;
#pragma unroll
  for (int q = 0; q < G / 32; ++q) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      uint32_t b[NT][4];
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr[j] + k0 + c * G + 32 * q + 8 * tig);
        b[j][0] = v.x; b[j][1] = v.y; b[j][2] = v.z; b[j][3] = v.w;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t a[4];
        if constexpr (std::is_same<OT, __half>::value) dequant_w4_word_f16(w[c][2 * q + h], a);
        else dequant_w4_word(w[c][2 * q + h], a);
#pragma unroll
        for (int j = 0; j < NT; ++j) mma16816<OT>(part[c][j], a, b[j][2 * h], b[j][2 * h + 1]);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const float2 s2 = bf162_to_f2(sc[c]);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      acc[j][0] = fmaf(part[c][j][0], s2.x, acc[j][0]);
      acc[j][1] = fmaf(part[c][j][1], s2.x, acc[j][1]);
      acc[j][2] = fmaf(part[c][j][2], s2.y, acc[j][2]);
      acc[j][3] = fmaf(part[c][j][3], s2.y, acc[j][3]);
    }
  }
}

// n consecutive chunks; NT = 2 n-tiles only when the unit has > 8 tokens.
template <int G>
__device__ __forceinline__ void w4_smem_run(const uint8_t* chunk, int n, const __half* const (&xr)[2], int k0, int lane,
                                       bool two, float (&acc)[2][4]) {
  constexpr int CHB = W4Fmt<G>::CHB;
  // one chunk per iteration: a small loop body (instruction fetch was the top stall with
  // two interleaved chunks, which gave no more issue parallelism)
  if (two) {
    for (int c = 0; c < n; ++c) w4_smem_chunks<G, 1, 2>(chunk + c * CHB, xr, k0 + c * G, lane, acc);
  } else {
    for (int c = 0; c < n; ++c) w4_smem_chunks<G, 1, 1>(chunk + c * CHB, xr, k0 + c * G, lane, acc);
  }
}

// acc[nt] += B16 chunk (16 rows x 64, in shared memory) . x rows (bf16 activations,
// permuted-K fragment order as the W4 chunks), accumulated like mma_frag (no scales).
template <int NT>
__device__ __forceinline__ void b16_smem_chunk(const uint8_t* chunk, const __nv_bfloat16* const (&xr)[2], int k0,
                                               int lane, float (&acc)[2][4]) {
  const int tig = lane & 3;
  uint32_t b[2][NT][4];
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr[j] + k0 + 32 * q + 8 * tig);
      b[q][j][0] = v.x; b[q][j][1] = v.y; b[q][j][2] = v.z; b[q][j][3] = v.w;
    }
#pragma unroll
  for (int st = 0; st < 4; ++st) {
    const uint4 u = *reinterpret_cast<const uint4*>(chunk + st * 512 + lane * 16);
    const uint32_t a[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < NT; ++j) mma16816<__nv_bfloat16>(acc[j], a, b[st >> 1][j][(st & 1) * 2], b[st >> 1][j][(st & 1) * 2 + 1]);
  }
}

// Fragment element r (0..3) of n-tile j: (row within the 16-row tile, token).
__device__ __forceinline__ int frag_row(int lane, int r) { return (lane >> 2) + 8 * (r >> 1); }
__device__ __forceinline__ int frag_tok(int lane, int j, int r) { return j * 8 + 2 * (lane & 3) + (r & 1); }

}  // namespace qw
