// Weight-streaming skinny GEMM core shared by the linear, MoE and lm_head kernels.
//
// y[t, n] = sum_k x[t, k] * W[n, k] for a handful of tokens t (a verify block) and a
// weight matrix streamed once from HBM.  The weight is the tensor-core A operand
// (16 output rows per warp tile), the tokens are the B operand (8 per n-tile), so one
// 128-bit weight load per lane feeds several mma.sync.m16n8k16 without any shared-
// memory round trip for the weights.  Weights are pre-packed ("streams") so that each
// lane's 16-byte loads are exactly its A fragments:
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
//   expert weights); fragments are gathered with 32-bit loads.
#pragma once

#include "qw_common.cuh"

namespace qw {

constexpr int SG_WARPS = 8;

template <int G>
struct W4Fmt {
  using ET = __nv_bfloat16;
  static constexpr int KCHUNK = G;
  static constexpr int STEPS = G / 16;
  static constexpr int WORDS = STEPS;              // 32-bit words per lane per chunk
  static constexpr int VW = STEPS < 4 ? STEPS : 4; // words per vector load
  static constexpr int NV = STEPS / VW;
  static constexpr int CHB = 8 * G + 32;
  static constexpr bool SCALED = true;

  // byte offset of row tile `rt` of a matrix with `k` columns (ld unused)
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
      } else if constexpr (VW == 2) {
        uint2 u = ldg_stream2(p);
        w[v * 2 + 0] = u.x; w[v * 2 + 1] = u.y;
      } else {
        w[v] = __ldg(reinterpret_cast<const uint32_t*>(p));
      }
    }
    sc = __ldg(reinterpret_cast<const uint32_t*>(chunk + 8 * G + (lane >> 2) * 4));
  }
  __device__ __forceinline__ static void afrag(const uint32_t (&w)[WORDS], int s, uint32_t (&a)[4]) {
    dequant_w4_word(w[s], a);
  }
};

struct B16Fmt {
  using ET = __nv_bfloat16;
  static constexpr int KCHUNK = 64;
  static constexpr int STEPS = 4;
  static constexpr int WORDS = 16;
  static constexpr int CHB = 2048;
  static constexpr bool SCALED = false;

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

// Row-major 16-bit matrix [N, K] with row stride `ld` bytes; K chunk of 16.
template <typename ET_>
struct RowFmt {
  using ET = ET_;
  static constexpr int KCHUNK = 16;
  static constexpr int STEPS = 1;
  static constexpr int WORDS = 4;
  static constexpr bool SCALED = false;

  __host__ __device__ static int64_t tile_offset(int64_t rt, int /*k*/, int64_t ld) {
    return rt * 16 * ld;
  }
  __device__ __forceinline__ static void load(const uint8_t* tile, int c, int lane, int64_t ld,
                                              uint32_t (&w)[WORDS], uint32_t& sc) {
    const int gid = lane >> 2, tig = lane & 3;
    const uint8_t* p = tile + static_cast<int64_t>(gid) * ld + (c * 16 + 2 * tig) * 2;
    w[0] = __ldg(reinterpret_cast<const uint32_t*>(p));
    w[1] = __ldg(reinterpret_cast<const uint32_t*>(p + 8 * ld));
    w[2] = __ldg(reinterpret_cast<const uint32_t*>(p + 16));
    w[3] = __ldg(reinterpret_cast<const uint32_t*>(p + 8 * ld + 16));
    sc = 0;
  }
  __device__ __forceinline__ static void afrag(const uint32_t (&w)[WORDS], int /*s*/, uint32_t (&a)[4]) {
    a[0] = w[0]; a[1] = w[1]; a[2] = w[2]; a[3] = w[3];
  }
};

// Accumulate one chunk of one 16-row weight tile against NT n-tiles (8 tokens each) of
// activations held in shared memory as xs[token][k].  `xs_lane` is this lane's
// ldmatrix.x4 row address for token block 0 at k = 0; token block j is `j * xstride16`
// elements further.
template <class Fmt, int NT>
__device__ __forceinline__ void mma_chunk(const uint32_t (&w)[Fmt::WORDS], uint32_t sc,
                                          const typename Fmt::ET* xs_lane, int xstride16, int kbase,
                                          float (&acc)[NT][4]) {
  using ET = typename Fmt::ET;
  if constexpr (Fmt::SCALED) {
    float part[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) part[j][0] = part[j][1] = part[j][2] = part[j][3] = 0.f;
#pragma unroll
    for (int s = 0; s < Fmt::STEPS; ++s) {
      uint32_t a[4];
      Fmt::afrag(w, s, a);
#pragma unroll
      for (int j = 0; j < NT / 2; ++j) {
        uint32_t b[4];
        ldmatrix_x4(b, xs_lane + j * xstride16 + kbase + s * 16);
        mma16816<ET>(part[2 * j], a, b[0], b[1]);
        mma16816<ET>(part[2 * j + 1], a, b[2], b[3]);
      }
    }
    const float2 s2 = bf162_to_f2(sc);  // (row gid, row gid + 8)
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
      Fmt::afrag(w, s, a);
#pragma unroll
      for (int j = 0; j < NT / 2; ++j) {
        uint32_t b[4];
        ldmatrix_x4(b, xs_lane + j * xstride16 + kbase + s * 16);
        mma16816<ET>(acc[2 * j], a, b[0], b[1]);
        mma16816<ET>(acc[2 * j + 1], a, b[2], b[3]);
      }
    }
  }
}

// Stream chunks [c0, c1) of one row tile with a PF-deep register prefetch ring.
template <class Fmt, int NT, int PF>
__device__ __forceinline__ void stream_tile(const uint8_t* tile, int64_t ld, int c0, int c1, int lane,
                                            const typename Fmt::ET* xs_lane, int xstride16,
                                            float (&acc)[NT][4]) {
  uint32_t w[PF][Fmt::WORDS];
  uint32_t sc[PF];
#pragma unroll
  for (int p = 0; p < PF; ++p)
    if (c0 + p < c1) Fmt::load(tile, c0 + p, lane, ld, w[p], sc[p]);
  for (int c = c0; c < c1; c += PF) {
#pragma unroll
    for (int p = 0; p < PF; ++p) {
      if (c + p < c1) {
        mma_chunk<Fmt, NT>(w[p], sc[p], xs_lane, xstride16, (c + p) * Fmt::KCHUNK, acc);
        if (c + p + PF < c1) Fmt::load(tile, c + p + PF, lane, ld, w[p], sc[p]);
      }
    }
  }
}

// Address of this lane's ldmatrix.x4 row for token block 0 (tokens 0..15) at k = 0.
template <typename ET>
__device__ __forceinline__ const ET* xs_lane_ptr(const ET* xs, int xstride, int lane) {
  const int tok = ((lane >> 4) << 3) + (lane & 7);
  const int kof = ((lane >> 3) & 1) << 3;
  return xs + tok * xstride + kof;
}

// Fragment element r (0..3) of n-tile j: (row within the 16-row tile, token).
__device__ __forceinline__ int frag_row(int lane, int r) { return (lane >> 2) + 8 * (r >> 1); }
__device__ __forceinline__ int frag_tok(int lane, int j, int r) { return j * 8 + 2 * (lane & 3) + (r & 1); }

}  // namespace qw
