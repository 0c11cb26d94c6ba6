// Layer-boundary kernels of the block verify: residual RMSNorm (with the embedding
// gather and the DFlash feature taps) and the acceptance step.
//
//  residual_norm  fused/model.py:398, :403, :407 — normed = round(round(h * rsqrt(mean h^2
//                 + eps)) * round(w + 1)) (zero-centred weights, :206-217); on the first
//                 layer h = embed[ids] (:346-347); a tap copies the residual stream after
//                 a feature layer (:405-406, target_features.py) into its feature slot, or
//                 the final-norm output when the tapped layer is the last (:407-409).
//  accept         the verify decision of fused/session.py:316-341 for a whole block:
//                 expected[0] = the pre-block prediction, expected[i] = argmax row i-1;
//                 proposal i is accepted while it equals expected[i].  The lm_head
//                 argmax keys are reduced here (ties -> lowest token id).
//  apply_commit   the bookkeeping of TargetVerification.commit (session.py:374-387):
//                 next prediction = row accepted-1 (or unchanged), position += accepted.
#include "qw_common.cuh"

namespace qw {

struct NormArgs {
  __nv_bfloat16* hidden;          // [T, H] residual stream (in/out)
  const int32_t* ids;             // [T] token ids, or null
  const __nv_bfloat16* embed;     // [V, H]
  const __nv_bfloat16* gamma;     // [H] zero-centred weight
  __nv_bfloat16* normed;          // [T, H]
  __nv_bfloat16* tap;             // feature slot base (row stride ldf), or null
  int64_t ldf;
  int tap_normed, T, H;
  float eps;
};

__global__ void residual_norm_kernel(NormArgs a) {
  __shared__ float red[32];
  constexpr int NV = 8;   // row values per thread held in registers (H <= NV * blockDim.x)
  const bool regs = a.H <= NV * static_cast<int>(blockDim.x);
  float g[NV];
  if (regs) {
    // the norm weight is no kernel's output: read before the wait
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = threadIdx.x + j * blockDim.x;
      g[j] = i < a.H ? rbf(__bfloat162float(a.gamma[i]) + 1.f) : 0.f;
    }
  }
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  __nv_bfloat16* h = a.hidden + static_cast<int64_t>(t) * a.H;
  if (a.ids) {
    const __nv_bfloat16* e = a.embed + static_cast<int64_t>(a.ids[t]) * a.H;
    for (int i = threadIdx.x; i < a.H; i += blockDim.x) h[i] = e[i];
    __syncthreads();
  }
  __nv_bfloat16* out = a.normed + static_cast<int64_t>(t) * a.H;
  __nv_bfloat16* tap = a.tap ? a.tap + static_cast<int64_t>(t) * a.ldf : nullptr;
  if (!regs) {
    rms_norm_row<false>(h, a.gamma, out, tap, a.tap_normed, a.H, a.eps, red);
    return;
  }
  // rms_norm_row's arithmetic with the row read once into registers
  __nv_bfloat16 hv[NV];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    hv[j] = i < a.H ? h[i] : __float2bfloat16_rn(0.f);
  }
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const float v = __bfloat162float(hv[j]);
    if (threadIdx.x + j * blockDim.x < a.H) ss += v * v;
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / a.H + a.eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < a.H) {
      const __nv_bfloat16 y = __float2bfloat16_rn(rbf(__bfloat162float(hv[j]) * inv) * g[j]);
      out[i] = y;
      if (tap) tap[i] = a.tap_normed ? y : hv[j];
    }
  }
}

// One CTA per token reduces its lm_head argmax keys; the CTA that finishes last (a
// ticket that wraps to 0 with the last token, so it is 0 again for the next launch;
// launches must not overlap) then evaluates acceptance for every sequence.
__device__ unsigned g_accept_ticket;

__global__ void accept_kernel(const unsigned long long* __restrict__ keys, int nblk, int T, int S, int B,
                              const int32_t* __restrict__ proposals, int32_t* __restrict__ top1,
                              int32_t* __restrict__ max_accepted, int32_t* __restrict__ next_token,
                              int32_t* __restrict__ accepted, int32_t* __restrict__ qpos, int auto_commit) {
  __shared__ unsigned long long s_best[32];
  __shared__ int s_last;
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  unsigned long long best = 0ull;
#pragma unroll 8
  for (int i = threadIdx.x; i < nblk; i += blockDim.x) {   // unrolled: the partial keys load together
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
    top1[t] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
    __threadfence();
    s_last = atomicInc(&g_accept_ticket, static_cast<unsigned>(T - 1)) == static_cast<unsigned>(T - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    int acc = 0;
    int expected = next_token[b];
    for (int i = 0; i < S; ++i) {
      if (proposals[b * S + i] != expected) break;
      ++acc;
      expected = __ldcg(top1 + b * S + i);
    }
    max_accepted[b] = acc;
    if (auto_commit) {
      accepted[b] = acc;
      if (acc > 0) next_token[b] = __ldcg(top1 + b * S + acc - 1);
      qpos[b] += acc;
    }
  }
}

__global__ void apply_commit_kernel(const int32_t* __restrict__ accepted, const int32_t* __restrict__ top1,
                                    int32_t* __restrict__ next_token, int32_t* __restrict__ qpos, int B, int S) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int acc = accepted[b];
  if (acc > 0) next_token[b] = top1[b * S + acc - 1];
  qpos[b] += acc;
}

}  // namespace qw

using namespace qw;

extern "C" int qw_residual_norm(void* hidden, const int32_t* ids, const void* embed, const void* gamma,
                                void* normed, void* tap, int64_t ldf, int tap_normed, int64_t tokens,
                                int64_t hidden_dim, float eps, void* stream) {
  QW_CHECK_ARG(hidden && gamma && normed && (ids == nullptr || embed != nullptr), "residual_norm: null pointer");
  QW_CHECK_ARG(tokens >= 0 && hidden_dim > 0 && eps > 0.f && (tap == nullptr || ldf >= hidden_dim),
               "residual_norm: invalid shape");
  if (tokens == 0) return QW_OK;
  NormArgs a{static_cast<__nv_bfloat16*>(hidden), ids, static_cast<const __nv_bfloat16*>(embed),
             static_cast<const __nv_bfloat16*>(gamma), static_cast<__nv_bfloat16*>(normed),
             static_cast<__nv_bfloat16*>(tap), ldf, tap_normed, static_cast<int>(tokens),
             static_cast<int>(hidden_dim), eps};
  QW_LAUNCH_PDL("residual_norm", residual_norm_kernel, dim3(static_cast<unsigned>(tokens)), dim3(256), 0,
                as_stream(stream), a);
  return QW_OK;
}

extern "C" int qw_accept(const void* keys, int64_t nblk, const int32_t* proposals, int32_t* top1,
                         int32_t* max_accepted, int32_t* next_token, int32_t* accepted, int32_t* qpos,
                         int64_t batch, int64_t seq, int auto_commit, void* stream) {
  QW_CHECK_ARG(keys && proposals && top1 && max_accepted && next_token, "accept: null pointer");
  QW_CHECK_ARG(!auto_commit || (accepted && qpos), "accept: auto commit needs accepted and qpos");
  QW_CHECK_ARG(batch >= 1 && seq >= 1 && seq <= QW_MAX_SEQ && batch * seq <= QW_MAX_BLOCK * 64 && nblk >= 1,
               "accept: invalid shape");
  QW_LAUNCH_PDL("accept", accept_kernel, dim3(static_cast<unsigned>(batch * seq)), dim3(256), 0, as_stream(stream),
                static_cast<const unsigned long long*>(keys), static_cast<int>(nblk),
                static_cast<int>(batch * seq), static_cast<int>(seq), static_cast<int>(batch), proposals, top1,
                max_accepted, next_token, accepted, qpos, auto_commit);
  return QW_OK;
}

extern "C" int qw_apply_commit(const int32_t* accepted, const int32_t* top1, int32_t* next_token, int32_t* qpos,
                               int64_t batch, int64_t seq, void* stream) {
  QW_CHECK_ARG(accepted && top1 && next_token && qpos && batch >= 1 && seq >= 1, "apply_commit: invalid argument");
  QW_LAUNCH_PDL("apply_commit", apply_commit_kernel, dim3(static_cast<unsigned>((batch + 127) / 128)), dim3(128), 0,
                as_stream(stream), accepted, top1, next_token, qpos, static_cast<int>(batch),
                static_cast<int>(seq));
  return QW_OK;
}
