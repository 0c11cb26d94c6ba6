// rms_norm, conv_state_update, causal_conv1d and cache_update of the fused-ops ABI
// (reference/fused_ops.py:28-56, :110-124).  HBM-bound data movement with fp32 math.
#include "qw_common.cuh"

namespace qw {

// ---------------------------------------------------------------- rms_norm
// One CTA per row; y = Ty(Tx(x * rsqrt(mean(x^2) + eps)) * gamma).
template <typename Tx, typename Tg, typename Ty>
__global__ void rms_norm_kernel(const Tx* __restrict__ x, const Tg* __restrict__ gamma,
                                Ty* __restrict__ y, int dim, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const Tx* xr = x + row * dim;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = to_f(xr[i]);
    ss += v * v;
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float n = rnd<Tx>(to_f(xr[i]) * inv);
    y[row * dim + i] = from_f<Ty>(n * to_f(gamma[i]));
  }
}

template <typename Tx, typename Tg, typename Ty>
static int launch_rms(const void* x, const void* g, void* y, int64_t rows, int64_t dim, float eps,
                      cudaStream_t s) {
  int threads = dim >= 1024 ? 256 : 128;
  rms_norm_kernel<Tx, Tg, Ty><<<static_cast<unsigned>(rows), threads, 0, s>>>(
      static_cast<const Tx*>(x), static_cast<const Tg*>(g), static_cast<Ty*>(y),
      static_cast<int>(dim), eps);
  QW_LAUNCH_CHECK("rms_norm");
  return QW_OK;
}

// ---------------------------------------------------------------- conv_state_update
// padded[b,c,i] = history[b,c,i] (i < K-1) else projected[b,i-(K-1),c];
// new_history[b,c,j] = padded[b,c,L-(K-1)+j].
template <typename T>
__global__ void conv_state_update_kernel(const T* __restrict__ proj, const T* __restrict__ hist,
                                         T* __restrict__ new_hist, T* __restrict__ padded,
                                         int64_t batch, int seq, int channels, int hk) {
  const int len = seq + hk;
  const int64_t total = batch * channels * static_cast<int64_t>(len);
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(idx % len);
    const int64_t bc = idx / len;
    const int c = static_cast<int>(bc % channels);
    const int64_t b = bc / channels;
    T v = i < hk ? hist[bc * hk + i] : proj[(b * seq + (i - hk)) * channels + c];
    padded[idx] = v;
    const int j = i - (len - hk);
    if (j >= 0) new_hist[bc * hk + j] = v;
  }
}

// ---------------------------------------------------------------- causal_conv1d
// out[b,t,c] = sum_j padded[b,c,t+j] * w[c,j]   (fp32 accumulate, one rounding)
template <typename T>
__global__ void causal_conv1d_kernel(const T* __restrict__ padded, const T* __restrict__ w,
                                     T* __restrict__ out, int64_t batch, int channels, int len,
                                     int kernel) {
  const int seq = len - kernel + 1;
  const int64_t total = batch * static_cast<int64_t>(seq) * channels;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % channels);
    const int64_t bt = idx / channels;
    const int t = static_cast<int>(bt % seq);
    const int64_t b = bt / seq;
    const T* p = padded + (b * channels + c) * len + t;
    float acc = 0.f;
    for (int j = 0; j < kernel; ++j) acc = fmaf(to_f(p[j]), to_f(w[c * kernel + j]), acc);
    out[idx] = from_f<T>(acc);
  }
}

// ---------------------------------------------------------------- cache_update
template <typename T>
__global__ void cache_concat_kernel(const T* __restrict__ old_k, const T* __restrict__ old_v,
                                    const T* __restrict__ new_k, const T* __restrict__ new_v,
                                    T* __restrict__ out_k, T* __restrict__ out_v, int64_t bh,
                                    int64_t t_old, int64_t t_new, int64_t dim) {
  const int64_t t_all = t_old + t_new;
  const int64_t total = bh * t_all * dim;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t d = idx % dim;
    const int64_t t = (idx / dim) % t_all;
    const int64_t r = idx / (dim * t_all);
    if (t < t_old) {
      out_k[idx] = old_k[(r * t_old + t) * dim + d];
      out_v[idx] = old_v[(r * t_old + t) * dim + d];
    } else {
      out_k[idx] = new_k[(r * t_new + (t - t_old)) * dim + d];
      out_v[idx] = new_v[(r * t_new + (t - t_old)) * dim + d];
    }
  }
}

static unsigned grid_for(int64_t total, int threads) {
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  return static_cast<unsigned>(blocks < 1 ? 1 : blocks);
}

}  // namespace qw

using namespace qw;

extern "C" int qw_rms_norm(const void* x, int x_dtype, const void* gamma, int gamma_dtype, void* y,
                           int y_dtype, int64_t rows, int64_t dim, float eps, void* stream) {
  QW_CHECK_ARG(x && gamma && y, "rms_norm: null pointer");
  QW_CHECK_ARG(rows >= 0 && dim > 0 && rows < (1LL << 31), "rms_norm: invalid shape");
  QW_CHECK_ARG(eps > 0.f, "RMSNorm needs positive epsilon and one gamma per feature");
  if (rows == 0) return QW_OK;
  cudaStream_t s = as_stream(stream);
  if (gamma_dtype == x_dtype && y_dtype == x_dtype) {
    switch (x_dtype) {
      case QW_F32: return launch_rms<float, float, float>(x, gamma, y, rows, dim, eps, s);
      case QW_F16: return launch_rms<__half, __half, __half>(x, gamma, y, rows, dim, eps, s);
      case QW_BF16:
        return launch_rms<__nv_bfloat16, __nv_bfloat16, __nv_bfloat16>(x, gamma, y, rows, dim, eps, s);
    }
  }
  if (gamma_dtype == QW_F32 && y_dtype == QW_F32) {
    switch (x_dtype) {
      case QW_F16: return launch_rms<__half, float, float>(x, gamma, y, rows, dim, eps, s);
      case QW_BF16: return launch_rms<__nv_bfloat16, float, float>(x, gamma, y, rows, dim, eps, s);
    }
  }
  return fail(QW_ERR_UNSUPPORTED, "rms_norm: unsupported dtype combination x=%d gamma=%d y=%d",
              x_dtype, gamma_dtype, y_dtype);
}

extern "C" int qw_conv_state_update(const void* projected, const void* history, void* new_history,
                                    void* padded, int dtype, int64_t batch, int64_t seq,
                                    int64_t channels, int64_t hist, void* stream) {
  QW_CHECK_ARG(projected && padded && (hist == 0 || (history && new_history)),
               "conv_state_update: null pointer");
  QW_CHECK_ARG(batch >= 0 && seq >= 1 && channels >= 1 && hist >= 0 && hist < 64,
               "conv state requires projected [B,S,C] and matching history [B,C,K-1]");
  if (batch == 0) return QW_OK;
  const int64_t total = batch * channels * (seq + hist);
  const unsigned grid = grid_for(total, 256);
  cudaStream_t s = as_stream(stream);
#define QW_CONV_UPD(T)                                                                     \
  conv_state_update_kernel<T><<<grid, 256, 0, s>>>(                                        \
      static_cast<const T*>(projected), static_cast<const T*>(history),                    \
      static_cast<T*>(new_history), static_cast<T*>(padded), batch, static_cast<int>(seq), \
      static_cast<int>(channels), static_cast<int>(hist))
  switch (dtype) {
    case QW_F32: QW_CONV_UPD(float); break;
    case QW_F16: QW_CONV_UPD(__half); break;
    case QW_BF16: QW_CONV_UPD(__nv_bfloat16); break;
    default: return fail(QW_ERR_ARG, "conv_state_update: bad dtype %d", dtype);
  }
#undef QW_CONV_UPD
  QW_LAUNCH_CHECK("conv_state_update");
  return QW_OK;
}

extern "C" int qw_causal_conv1d(const void* padded, const void* weight, void* out, int dtype,
                                int64_t batch, int64_t channels, int64_t padded_len, int64_t kernel,
                                void* stream) {
  QW_CHECK_ARG(padded && weight && out, "causal_conv1d: null pointer");
  QW_CHECK_ARG(batch >= 0 && channels >= 1 && kernel >= 1 && padded_len >= kernel,
               "depthwise conv requires [B,C,S+K-1] and [C,1,K]");
  if (batch == 0) return QW_OK;
  const int64_t total = batch * channels * (padded_len - kernel + 1);
  const unsigned grid = grid_for(total, 256);
  cudaStream_t s = as_stream(stream);
#define QW_CONV(T)                                                                             \
  causal_conv1d_kernel<T><<<grid, 256, 0, s>>>(static_cast<const T*>(padded),                   \
                                               static_cast<const T*>(weight), static_cast<T*>(out), \
                                               batch, static_cast<int>(channels),              \
                                               static_cast<int>(padded_len), static_cast<int>(kernel))
  switch (dtype) {
    case QW_F32: QW_CONV(float); break;
    case QW_F16: QW_CONV(__half); break;
    case QW_BF16: QW_CONV(__nv_bfloat16); break;
    default: return fail(QW_ERR_ARG, "causal_conv1d: bad dtype %d", dtype);
  }
#undef QW_CONV
  QW_LAUNCH_CHECK("causal_conv1d");
  return QW_OK;
}

extern "C" int qw_cache_update(const void* key, const void* value, const void* new_key,
                               const void* new_value, void* out_key, void* out_value, int dtype,
                               int64_t batch, int64_t kv_heads, int64_t t_old, int64_t t_new,
                               int64_t dim, void* stream) {
  QW_CHECK_ARG(new_key && new_value && out_key && out_value, "cache_update: null pointer");
  QW_CHECK_ARG(t_old == 0 || (key && value), "KV caches must appear together and use [B,H,T,D]");
  QW_CHECK_ARG(batch >= 0 && kv_heads >= 1 && t_old >= 0 && t_new >= 0 && dim >= 1,
               "cache_update: invalid shape");
  const int64_t total = batch * kv_heads * (t_old + t_new) * dim;
  if (total == 0) return QW_OK;
  const unsigned grid = grid_for(total, 256);
  cudaStream_t s = as_stream(stream);
#define QW_CAT(T)                                                                              \
  cache_concat_kernel<T><<<grid, 256, 0, s>>>(                                                 \
      static_cast<const T*>(key), static_cast<const T*>(value), static_cast<const T*>(new_key), \
      static_cast<const T*>(new_value), static_cast<T*>(out_key), static_cast<T*>(out_value),  \
      batch * kv_heads, t_old, t_new, dim)
  switch (dtype) {
    case QW_F32: QW_CAT(float); break;
    case QW_F16: QW_CAT(__half); break;
    case QW_BF16: QW_CAT(__nv_bfloat16); break;
    default: return fail(QW_ERR_ARG, "cache_update: bad dtype %d", dtype);
  }
#undef QW_CAT
  QW_LAUNCH_CHECK("cache_update");
  return QW_OK;
}
