// Streaming linear y = x . W^T for the verify block's tokens (W4A16 or bf16 weights).
// Replaces the quantised / dense projections of fused/model.py:197-204 and
// fused/quantization.py:154-165.  HBM-bound: each weight byte is read once per
// 32-token pass; the CTA splits K across its warps and reduces in shared memory, so
// the result is deterministic and the epilogue can fuse the residual add.
#include <mutex>

#include "stream_gemm.cuh"

namespace qw {

struct LinArgs {
  const __nv_bfloat16* x;  // [T, k]
  const uint8_t* w;        // stream
  void* y;                 // [T, ldy] (argmax: optional bf16 logits)
  int64_t ldy;
  int tokens, n, k, rt, mode;
  unsigned long long* keys;  // argmax: [gridDim.x, tokens] best (value, index) key per CTA
};

// Argmax key of logit `v` (rounded to bf16, the reference's logits dtype) at row n:
// larger value wins, then the lower index (torch argmax returns the first maximum).
__device__ __forceinline__ unsigned long long argmax_key(float v, int n) {
  return (static_cast<unsigned long long>(float_key(rbf(v))) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(n));
}

template <class Fmt, int NT, int PF, bool ARGMAX = false>
__global__ void __launch_bounds__(SG_WARPS * 32) stream_linear_kernel(LinArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int NTOK = NT * 8;
  float* red = reinterpret_cast<float*>(smem);  // [SG_WARPS][NT*4][32]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KS = SG_WARPS / a.rt;
  const int rt_local = warp / KS, ks = warp % KS;
  const int ntiles = a.n / 16;
  const int rt = blockIdx.x * a.rt + rt_local;
  const bool active = rt < ntiles;
  const int nch = a.k / Fmt::KCHUNK;
  const int c0 = ks * nch / KS, c1 = (ks + 1) * nch / KS;
  const uint8_t* tile = a.w + Fmt::tile_offset(active ? rt : 0, a.k, 0);
  const int gid = lane >> 2, tig = lane & 3;

  for (int tp0 = 0; tp0 < a.tokens; tp0 += NTOK) {
    XRows<__nv_bfloat16, NT> xr;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int t = min(tp0 + j * 8 + gid, a.tokens - 1);  // rows past the last token: any valid row
      xr.r[j] = a.x + static_cast<int64_t>(t) * a.k;
    }
    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    if (active) stream_tile<Fmt, NT, PF, true>(tile, 0, c0, c1, lane, xr, acc);
    pdl_wait();                    // (idle warps) before any write of this kernel
    pdl_trigger();
    if (tp0 > 0) __syncthreads();  // previous pass's reduction reads are done
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) red[(warp * NT * 4 + j * 4 + r) * 32 + lane] = acc[j][r];
    __syncthreads();
    if constexpr (ARGMAX) {
      // per-token best over this CTA's rows: lanes hold (row gid / gid+8, token), reduce
      // over gid with shuffles, then across the CTA's row tiles in shared memory
      unsigned long long* best = reinterpret_cast<unsigned long long*>(red + SG_WARPS * NT * 4 * 32);
      if (ks == 0) {
#pragma unroll
        for (int j = 0; j < NT; ++j) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // token parity (r & 1)
            unsigned long long key = 0ull;
            const int t = tp0 + j * 8 + 2 * tig + h;
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
              const int r = rr * 2 + h;
              float v = 0.f;
              for (int s = 0; s < KS; ++s) v += red[((warp + s) * NT * 4 + j * 4 + r) * 32 + lane];
              const int n = rt * 16 + gid + 8 * rr;
              if (active && t < a.tokens) {
                const unsigned long long kk = argmax_key(v, n);
                key = kk > key ? kk : key;
                if (a.y) static_cast<__nv_bfloat16*>(a.y)[static_cast<int64_t>(t) * a.ldy + n] = __float2bfloat16_rn(v);
              }
            }
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
              const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
              key = other > key ? other : key;
            }
            if (gid == 0) best[rt_local * NTOK + j * 8 + 2 * tig + h] = key;
          }
        }
      }
      __syncthreads();
      if (threadIdx.x < NTOK && tp0 + threadIdx.x < a.tokens) {
        unsigned long long key = 0ull;
        for (int r = 0; r < a.rt; ++r) {
          const unsigned long long kk = best[r * NTOK + threadIdx.x];
          key = kk > key ? kk : key;
        }
        a.keys[static_cast<int64_t>(blockIdx.x) * a.tokens + tp0 + threadIdx.x] = key;
      }
    } else if (ks == 0 && active) {
#pragma unroll
      for (int j = 0; j < NT; ++j) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float v = 0.f;
          for (int s = 0; s < KS; ++s) v += red[((warp + s) * NT * 4 + j * 4 + r) * 32 + lane];
          const int t = tp0 + j * 8 + 2 * tig + (r & 1);
          const int n = rt * 16 + gid + 8 * (r >> 1);
          if (t < a.tokens) {
            const int64_t o = static_cast<int64_t>(t) * a.ldy + n;
            if (a.mode == QW_OUT_F32) {
              static_cast<float*>(a.y)[o] = v;
            } else if (a.mode == QW_OUT_BF16) {
              static_cast<__nv_bfloat16*>(a.y)[o] = __float2bfloat16_rn(v);
            } else {
              __nv_bfloat16* y = static_cast<__nv_bfloat16*>(a.y);
              y[o] = __float2bfloat16_rn(__bfloat162float(y[o]) + rbf(v));
            }
          }
        }
      }
    }
  }
}

// Row tiles per CTA (the K split is SG_WARPS / rt): the largest count that still leaves
// >= 2 waves of CTAs.  The partition (and so the fp32 summation order) depends on the
// weight shape only, never on the token count, so a token's output has the same bits
// whichever block size computes it.
static int choose_rt(int ntiles) {
  for (int rt : {8, 4, 2}) {
    if ((ntiles + rt - 1) / rt >= 296) return rt;
  }
  return 1;
}

template <class Fmt, int NT, int PF, bool ARGMAX = false>
static int launch_linear(const LinArgs& a0, cudaStream_t s) {
  LinArgs a = a0;
  if (a.rt <= 0) a.rt = choose_rt(a.n / 16);
  const size_t smem = SG_WARPS * NT * 4 * 32 * 4 + (ARGMAX ? SG_WARPS * NT * 8 * 8 : 0);
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(stream_linear_kernel<Fmt, NT, PF, ARGMAX>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (attr_err != cudaSuccess) return cuda_status(attr_err, "linear smem attribute");
  const int ntiles = a.n / 16;
  const unsigned grid = static_cast<unsigned>((ntiles + a.rt - 1) / a.rt);
  QW_LAUNCH_PDL("linear", stream_linear_kernel<Fmt, NT, PF, ARGMAX>, dim3(grid), dim3(SG_WARPS * 32), smem, s, a);
  return QW_OK;
}

template <class Fmt, int PF>
static int dispatch_nt(const LinArgs& a, cudaStream_t s) {
  if (a.tokens > 16) return launch_linear<Fmt, 4, PF>(a, s);
  return launch_linear<Fmt, 2, PF>(a, s);
}

static int check_linear(const void* x, const void* w, void* y, int mode, int64_t ldy,
                        int64_t tokens, int64_t n, int64_t k) {
  QW_CHECK_ARG(x && w && y, "linear: null pointer");
  QW_CHECK_ARG(tokens >= 0 && tokens < (1 << 24), "linear: bad token count");
  QW_CHECK_ARG(n > 0 && n % 16 == 0 && n < (1LL << 30), "linear: N must be a positive multiple of 16");
  QW_CHECK_ARG(k > 0 && k < (1 << 20), "linear: bad K");
  QW_CHECK_ARG(ldy >= n, "linear: ldy < N");
  QW_CHECK_ARG(mode == QW_OUT_BF16 || mode == QW_OUT_F32 || mode == QW_OUT_RESID_BF16,
               "linear: bad output mode");
  QW_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0,
               "linear: x and w must be 16-byte aligned");
  QW_CHECK_ARG(k % 32 == 0, "linear: K must be a multiple of 32");
  return QW_OK;
}

}  // namespace qw

using namespace qw;

extern "C" int64_t qw_w4_stream_bytes(int64_t n, int64_t k, int32_t group) {
  if (n <= 0 || k <= 0 || n % 16 || (group != 32 && group != 64 && group != 128) || k % group) return -1;
  return (n / 16) * (k / group) * (8LL * group + 32);
}

extern "C" int64_t qw_b16_stream_bytes(int64_t n, int64_t k) {
  if (n <= 0 || k <= 0 || n % 16 || k % 64) return -1;
  return (n / 16) * (k / 64) * 2048LL;
}

extern "C" int qw_w4_linear(const void* x, const void* w_stream, void* y, int mode, int64_t ldy,
                            int64_t tokens, int64_t n, int64_t k, int32_t group, void* stream) {
  int st = check_linear(x, w_stream, y, mode, ldy, tokens, n, k);
  if (st) return st;
  QW_CHECK_ARG(group == 32 || group == 64 || group == 128, "w4_linear: group must be 32, 64 or 128");
  QW_CHECK_ARG(k % group == 0, "w4_linear: K %% group != 0");
  if (tokens == 0) return QW_OK;
  LinArgs a{static_cast<const __nv_bfloat16*>(x), static_cast<const uint8_t*>(w_stream), y, ldy,
            static_cast<int>(tokens), static_cast<int>(n), static_cast<int>(k), 0, mode};
  cudaStream_t s = as_stream(stream);
  switch (group) {
    case 128: return dispatch_nt<W4Fmt<128>, 4>(a, s);
    case 64: return dispatch_nt<W4Fmt<64>, 4>(a, s);
    default: return dispatch_nt<W4Fmt<32>, 4>(a, s);
  }
}

extern "C" int qw_b16_linear(const void* x, const void* w_stream, void* y, int mode, int64_t ldy,
                             int64_t tokens, int64_t n, int64_t k, void* stream) {
  int st = check_linear(x, w_stream, y, mode, ldy, tokens, n, k);
  if (st) return st;
  QW_CHECK_ARG(k % 64 == 0, "b16_linear: K must be a multiple of 64");
  if (tokens == 0) return QW_OK;
  LinArgs a{static_cast<const __nv_bfloat16*>(x), static_cast<const uint8_t*>(w_stream), y, ldy,
            static_cast<int>(tokens), static_cast<int>(n), static_cast<int>(k), 0, mode};
  return dispatch_nt<B16Fmt, 4>(a, as_stream(stream));
}

// The lm_head streams 8 row tiles per CTA (each warp a whole tile, all of K): fewer
// argmax partials per token for the accept reduction.
constexpr int LMHEAD_RT = 8;

extern "C" int64_t qw_lmhead_blocks(int64_t n) {
  if (n <= 0 || n % 16) return -1;
  return (n / 16 + LMHEAD_RT - 1) / LMHEAD_RT;
}

extern "C" int qw_lmhead_argmax(const void* x, const void* w_stream, void* logits, void* keys, int64_t tokens,
                                int64_t n, int64_t k, void* stream) {
  int st = check_linear(x, w_stream, keys, QW_OUT_BF16, n, tokens, n, k);
  if (st) return st;
  QW_CHECK_ARG(k % 64 == 0, "lmhead: K must be a multiple of 64");
  if (tokens == 0) return QW_OK;
  LinArgs a{static_cast<const __nv_bfloat16*>(x), static_cast<const uint8_t*>(w_stream), logits, n,
            static_cast<int>(tokens), static_cast<int>(n), static_cast<int>(k), LMHEAD_RT, QW_OUT_BF16,
            static_cast<unsigned long long*>(keys)};
  return launch_linear<B16Fmt, 2, 4, true>(a, as_stream(stream));
}
