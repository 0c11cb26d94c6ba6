// Kernels of the DFlash draft forward (model/qwen35_moe_dflash/model.py:102-522, the
// draft graph's block and context construction model/qwen35_moe_dflash/reference/
// graphs.py:63-97) that the verify path's kernels do not already cover.  The draft's
// projections run on the bf16 streaming linears, its norms on the RMSNorm operator and
// its attention on the paged attention kernels with the draft's masks.
//
//  draft_prep     q/k RMSNorm with the draft's effective weights (ops.py:66-71), rotary
//                 over the whole head (model.py:80-99, ops.py:75-90; fp32 angles, cos/sin
//                 rounded to bf16), and the append of k/v into the draft's paged cache.
//                 Used twice per step: for the committed rows of the last verify block
//                 (the context the draft attends to: k/v only, rows below the accepted
//                 count, at their positions) and for the draft block itself (q, k, v).
//  swiglu         silu(gate) * up with the reference's bf16 rounding points.
//  block_embed    the block [anchor, mask, ..., mask] through the shared embedding.
//  propose        the arg-max of the lm_head keys of rows 1 .. S-1 (ties -> lowest id)
//                 written as the next verify block [anchor, proposals...].
#include "qw_common.cuh"

namespace qw {

constexpr int DP_THREADS = 128;

template <int D>
__global__ void __launch_bounds__(DP_THREADS) draft_prep_kernel(
    const __nv_bfloat16* __restrict__ qkv, int64_t ldq, int has_q, const __nv_bfloat16* __restrict__ qn_w,
    const __nv_bfloat16* __restrict__ kn_w, float eps, float theta, const int32_t* __restrict__ pos_base,
    const int32_t* __restrict__ pos_sub, const int32_t* __restrict__ valid, const int32_t* __restrict__ pages,
    int max_pages, int P, __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc,
    __nv_bfloat16* __restrict__ qout, int S, int H, int Hkv) {
  constexpr int NPT = (D + DP_THREADS - 1) / DP_THREADS;
  __shared__ float red[32];
  __shared__ float xr[D];
  const int t = blockIdx.x;
  const int b = t / S, s = t % S;
  const int slot = blockIdx.y;
  const bool is_q = has_q && slot < H;
  const int head = is_q ? slot : slot - (has_q ? H : 0);
  const __nv_bfloat16* gw = is_q ? qn_w : kn_w;
  float gpre[NPT], inv_freq[NPT];
#pragma unroll
  for (int j = 0; j < NPT; ++j) {
    const int d = threadIdx.x + j * DP_THREADS;
    gpre[j] = d < D ? __bfloat162float(gw[d]) : 0.f;   // the effective scale (no +1)
    inv_freq[j] = 1.0f / powf(theta, static_cast<float>(2 * (d % (D / 2))) / D);
  }
  pdl_wait();   // qkv from the projection; positions and counts from earlier kernels
  pdl_trigger();
  if (valid && s >= valid[b]) return;   // a row past the committed count: nothing to append
  const int pos = pos_base[b] - (pos_sub ? pos_sub[b] : 0) + s;
  const int kofs = has_q ? H * D : 0;
  const __nv_bfloat16* src = qkv + t * ldq + (is_q ? head * D : kofs + head * D);
  float xv[NPT];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NPT; ++j) {
    const int d = threadIdx.x + j * DP_THREADS;
    xv[j] = d < D ? __bfloat162float(src[d]) : 0.f;
    ss += xv[j] * xv[j];
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / D + eps);
#pragma unroll
  for (int j = 0; j < NPT; ++j) {
    const int d = threadIdx.x + j * DP_THREADS;
    if (d < D) xr[d] = rbf(rbf(xv[j] * inv) * gpre[j]);
  }
  __syncthreads();
  const int page = is_q ? 0 : pages[b * max_pages + pos / P];
#pragma unroll
  for (int j = 0; j < NPT; ++j) {
    const int d = threadIdx.x + j * DP_THREADS;
    if (d >= D) continue;
    const float ang = static_cast<float>(pos) * inv_freq[j];
    const float other = d < D / 2 ? -xr[d + D / 2] : xr[d - D / 2];
    const float y = rbf(rbf(xr[d] * rbf(cosf(ang))) + rbf(other * rbf(sinf(ang))));
    if (is_q) {
      qout[((static_cast<int64_t>(b) * H + head) * S + s) * D + d] = __float2bfloat16_rn(y);
    } else {
      const int64_t off = ((static_cast<int64_t>(page) * Hkv + head) * P + pos % P) * D + d;
      kc[off] = __float2bfloat16_rn(y);
      vc[off] = qkv[t * ldq + kofs + Hkv * D + head * D + d];
    }
  }
}

__global__ void swiglu_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out, int T, int I) {
  pdl_wait();
  pdl_trigger();
  const int64_t n = static_cast<int64_t>(T) * I;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / I, c = i % I;
    const float g = __bfloat162float(gu[t * 2 * I + c]), u = __bfloat162float(gu[t * 2 * I + I + c]);
    out[i] = __float2bfloat16_rn(rbf(silu_f(g)) * u);
  }
}

__global__ void block_embed_kernel(const __nv_bfloat16* __restrict__ embed, const int32_t* __restrict__ anchor,
                                   int mask_id, __nv_bfloat16* __restrict__ hidden, int S, int H) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x, b = t / S, s = t % S;
  const int64_t id = s == 0 ? anchor[b] : mask_id;
  const uint4* src = reinterpret_cast<const uint4*>(embed + id * H);
  uint4* dst = reinterpret_cast<uint4*>(hidden + static_cast<int64_t>(t) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// One CTA per block row: row 0 takes the anchor, row i >= 1 the arg-max of its lm_head
// keys (value key above 0xFFFFFFFF - id: the lowest id wins a tie).
__global__ void propose_kernel(const unsigned long long* __restrict__ keys, int nblk, int T, int S,
                               const int32_t* __restrict__ anchor, int32_t* __restrict__ tokens) {
  __shared__ unsigned long long s_best[32];
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x, b = t / S, s = t % S;
  if (s == 0) {
    if (threadIdx.x == 0) tokens[t] = anchor[b];
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < nblk; i += blockDim.x) {
    const unsigned long long k = keys[static_cast<int64_t>(i) * T + t];
    best = k > best ? k : best;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if (lane == 0) s_best[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < nw; ++w) best = s_best[w] > best ? s_best[w] : best;
    tokens[t] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
  }
}

}  // namespace qw

using namespace qw;

extern "C" int qw_draft_prep(const void* qkv, int64_t ldq, int has_q, const void* q_norm_w, const void* k_norm_w,
                             float eps, float rope_theta, const int32_t* pos_base, const int32_t* pos_sub,
                             const int32_t* valid, const int32_t* pages, int32_t max_pages, int32_t page_size,
                             void* k_cache, void* v_cache, void* q_out, int64_t batch, int64_t seq, int64_t heads,
                             int64_t kv_heads, int64_t dim, void* stream) {
  QW_CHECK_ARG(qkv && k_norm_w && pos_base && pages && k_cache && v_cache && (!has_q || (q_norm_w && q_out)),
               "draft_prep: null pointer");
  QW_CHECK_ARG(batch >= 1 && seq >= 1 && heads >= 1 && kv_heads >= 1 && page_size >= 1 && max_pages >= 1 &&
                   ldq >= (has_q ? heads : 0) * dim + 2 * kv_heads * dim && (has_q == 0 || has_q == 1),
               "draft_prep: invalid shape");
  const dim3 grid(static_cast<unsigned>(batch * seq), static_cast<unsigned>((has_q ? heads : 0) + kv_heads));
  cudaStream_t st = as_stream(stream);
#define QW_DPREP(DD)                                                                                          \
  QW_LAUNCH_PDL("draft_prep", draft_prep_kernel<DD>, grid, dim3(DP_THREADS), 0, st,                           \
                static_cast<const __nv_bfloat16*>(qkv), ldq, has_q, static_cast<const __nv_bfloat16*>(q_norm_w),  \
                static_cast<const __nv_bfloat16*>(k_norm_w), eps, rope_theta, pos_base, pos_sub, valid, pages, \
                max_pages, page_size, static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), \
                static_cast<__nv_bfloat16*>(q_out), static_cast<int>(seq), static_cast<int>(heads),             \
                static_cast<int>(kv_heads))
  switch (dim) {
    case 64: QW_DPREP(64); break;
    case 128: QW_DPREP(128); break;
    case 256: QW_DPREP(256); break;
    default: return fail(QW_ERR_UNSUPPORTED, "draft_prep: head dim %lld not built", static_cast<long long>(dim));
  }
#undef QW_DPREP
  return QW_OK;
}

extern "C" int qw_swiglu(const void* gate_up, void* out, int64_t tokens, int64_t inter, void* stream) {
  QW_CHECK_ARG(gate_up && out && tokens >= 1 && inter >= 1, "swiglu: invalid argument");
  const int64_t n = tokens * inter;
  const unsigned grid = static_cast<unsigned>((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184);
  QW_LAUNCH_PDL("swiglu", swiglu_kernel, dim3(grid), dim3(256), 0, as_stream(stream),
                static_cast<const __nv_bfloat16*>(gate_up), static_cast<__nv_bfloat16*>(out), static_cast<int>(tokens),
                static_cast<int>(inter));
  return QW_OK;
}

extern "C" int qw_draft_block_embed(const void* embed, const int32_t* anchor, int32_t mask_id, void* hidden,
                                    int64_t batch, int64_t seq, int64_t hidden_dim, void* stream) {
  QW_CHECK_ARG(embed && anchor && hidden && batch >= 1 && seq >= 1 && hidden_dim % 8 == 0 && mask_id >= 0,
               "draft_block_embed: invalid argument");
  QW_LAUNCH_PDL("draft_block_embed", block_embed_kernel, dim3(static_cast<unsigned>(batch * seq)), dim3(128), 0,
                as_stream(stream), static_cast<const __nv_bfloat16*>(embed), anchor, mask_id,
                static_cast<__nv_bfloat16*>(hidden), static_cast<int>(seq), static_cast<int>(hidden_dim));
  return QW_OK;
}

extern "C" int qw_draft_propose(const void* keys, int64_t nblk, const int32_t* anchor, int32_t* tokens,
                                int64_t batch, int64_t seq, void* stream) {
  QW_CHECK_ARG(keys && anchor && tokens && nblk >= 1 && batch >= 1 && seq >= 2, "draft_propose: invalid argument");
  QW_LAUNCH_PDL("draft_propose", propose_kernel, dim3(static_cast<unsigned>(batch * seq)), dim3(256), 0,
                as_stream(stream), static_cast<const unsigned long long*>(keys), static_cast<int>(nblk),
                static_cast<int>(batch * seq), static_cast<int>(seq), anchor, tokens);
  return QW_OK;
}
