// Shared device/host helpers for the sm_100a kernels of libqw_b200.
#pragma once

#include <mutex>

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>
#include <type_traits>
#include <utility>

#include "../../include/qw_b200.h"

namespace qw {

// ------------------------------------------------------------------ host-side status
void set_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);
int cuda_status(cudaError_t err, const char* what);

// Bounded device waits (bulk-copy rings) record an expiry in a sticky word of their
// translation unit; these return that word's device address on the current device.
int linear_wait_status_addr(int32_t** out);
int moe_wait_status_addr(int32_t** out);

// Test-only injection into the cluster linear kernels' waits (qw_debug_inject_wait_timeout):
// the wait limit in cycles (0: the default) and extra bytes announced on every stage's
// barrier beyond the bytes copied, so that no stage completes and every wait expires.
struct WaitInjection {
  long long limit;
  unsigned tx_excess;
};
WaitInjection wait_injection();

// Device address of a __device__ variable on the current device, looked up once per
// device (cudaGetSymbolAddress with that device current) and cached.  `sym` must be
// named in the translation unit that defines it.
template <typename T>
int symbol_addr_cached(const T& sym, T** cache, int ncache, std::mutex& mu, T** out, const char* what) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_status(err, what);
  if (dev < 0 || dev >= ncache) return fail(QW_ERR_UNSUPPORTED, "%s: device %d beyond the %d tracked", what, dev, ncache);
  std::lock_guard<std::mutex> guard(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, sym);
    if (err != cudaSuccess) return cuda_status(err, what);
    cache[dev] = static_cast<T*>(p);
  }
  *out = cache[dev];
  return QW_OK;
}

#define QW_CHECK_ARG(cond, ...)                                   \
  do {                                                            \
    if (!(cond)) return ::qw::fail(QW_ERR_ARG, __VA_ARGS__);      \
  } while (0)

#define QW_LAUNCH_CHECK(what)                                                      \
  do {                                                                             \
    cudaError_t _e = cudaGetLastError();                                           \
    if (_e != cudaSuccess) return ::qw::cuda_status(_e, what);                     \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ------------------------------------------------------------------ programmatic launch
// Kernels of the verify step are launched with programmatic stream serialization: a
// kernel may start while its predecessor on the stream drains, runs its independent
// prologue (weights, which no kernel writes; data of kernels before the predecessor),
// then pdl_wait() blocks until the predecessor has completed and its writes are
// visible.  pdl_trigger() (only after pdl_wait) lets the successor start early in turn.
// Without a programmatic predecessor both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// Split cluster barrier.  Every thread of every CTA of the cluster arrives (relaxed: it
// publishes no memory) and later waits; after the wait every CTA of the cluster is known
// to be running, which distributed shared memory stores into a peer CTA require.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

#define QW_LAUNCH_PDL(what, ...)                                                  \
  do {                                                                            \
    cudaError_t _e = ::qw::launch_pdl(__VA_ARGS__);                               \
    if (_e != cudaSuccess) return ::qw::cuda_status(_e, what);                    \
  } while (0)

// ------------------------------------------------------------------ dtype helpers
template <typename T> struct DT;
template <> struct DT<float> { static constexpr int id = QW_F32; };
template <> struct DT<__half> { static constexpr int id = QW_F16; };
template <> struct DT<__nv_bfloat16> { static constexpr int id = QW_BF16; };

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Round a float to the value the storage type T would hold (the reference's torch ops
// return tensors of the activation dtype at these points).
template <typename T> __device__ __forceinline__ float rnd(float x) { return to_f(from_f<T>(x)); }
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// SiLU and sigmoid with the fast reciprocal-multiply division (within 2 ulp of the
// correctly rounded quotient, far below the bf16 rounding that follows every use): the
// IEEE division sequence dominated the GDN conv prologue.  __fdividef returns 0 when the
// denominator exceeds 2^126 (x < -87), where both functions are 0 to float precision
// after rounding.
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x <= 1024; `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
  if (warp == 0) {
    t = warp_sum(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

// RMSNorm of one token's row with the +1 gamma convention of qw_residual_norm:
// out = bf16(bf16(h * rsqrt(mean(h^2) + eps)) * bf16(gamma + 1)), and the feature tap
// (h, or out with tap_normed) when tap != null.  Every thread of the CTA calls it; the
// same thread count gives the same bits.  CG: h was written by other CTAs of this
// launch, so it is read through L2 only.
template <bool CG>
__device__ __forceinline__ void rms_norm_row(const __nv_bfloat16* h, const __nv_bfloat16* gamma, __nv_bfloat16* out,
                                             __nv_bfloat16* tap, int tap_normed, int H, float eps, float* red) {
  float ss = 0.f;
#pragma unroll 8
  for (int i = threadIdx.x; i < H; i += blockDim.x) {   // unrolled: the row loads are in flight together
    const float v = __bfloat162float(CG ? __ldcg(h + i) : h[i]);
    ss += v * v;
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / H + eps);
#pragma unroll 8
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const __nv_bfloat16 hv = CG ? __ldcg(h + i) : h[i];
    const float g = rbf(__bfloat162float(gamma[i]) + 1.f);
    const __nv_bfloat16 y = __float2bfloat16_rn(rbf(__bfloat162float(hv) * inv) * g);
    out[i] = y;
    if (tap) tap[i] = tap_normed ? y : hv;
  }
}

// ------------------------------------------------------------------ tensor-core helpers
// mma.sync m16n8k16 bf16 x bf16 -> f32 (row.col).  A: 4 x b32, B: 2 x b32, C/D: 4 x f32.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// fp16 variant (same fragment layout).
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename ET>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<ET, __half>::value) {
    mma_f16_16816(d, a, b0, b1);
  } else {
    mma_bf16_16816(d, a, b0, b1);
  }
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* smem_row) {
  uint32_t addr = static_cast<uint32_t>(__cvta_generic_to_shared(smem_row));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x2(uint32_t (&r)[2], const void* smem_row) {
  uint32_t addr = static_cast<uint32_t>(__cvta_generic_to_shared(smem_row));
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* smem_row) {
  uint32_t addr = static_cast<uint32_t>(__cvta_generic_to_shared(smem_row));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Streaming 128-bit global load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg_stream2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}

// 16-byte asynchronous global -> shared copy (L2 only); when !valid the destination
// is zero-filled and nothing is read (src must still be a mapped address).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));  // (a & b) | c
  return d;
}

// One 32-bit word of the W4 stream holds 8 offset-binary nibbles u = q + 8.  Nibble j of
// the word and nibble j+4 land in the two bf16 halves of A-fragment register j (j<4):
// OR-ing the nibble into the mantissa of bf16 128.0 (0x4300) gives 128 + u exactly;
// subtracting 136 leaves q as an exact bf16 integer.
__device__ __forceinline__ void dequant_w4_word(uint32_t w, uint32_t (&a)[4]) {
  const uint32_t MASK = 0x000F000Fu, EXP = 0x43004300u;
  const __nv_bfloat162 off = __floats2bfloat162_rn(136.f, 136.f);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t r = lop3_and_or(w >> (4 * j), MASK, EXP);
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&r);
    v = __hsub2(v, off);
    a[j] = *reinterpret_cast<uint32_t*>(&v);
  }
}

// The same word as fp16 A fragments with no arithmetic at all: each fp16 lane keeps its
// stored nibble n in place, so nibbles 0, 2 (bits 0-3 of a half) read as the subnormal
// n * 2^-24 and nibbles 1, 3 (bits 4-7) as n * 2^-20 -- exact values the MMA multiplies
// exactly.  Register j holds nibbles (j, j + 4) as in dequant_w4_word_f16, so registers
// 0, 2 (A rows gid) carry the 2^-24 lanes and registers 1, 3 (rows gid + 8) the 2^-20
// lanes; the caller restores q = n - 8 per row from the MMA sum P and the activation
// sum X of the same k range: sum (n - 8) x = 2^24 P - 8 X (rows gid), 2^20 P - 8 X
// (rows gid + 8).
__device__ __forceinline__ void w4_nibbles_f16(uint32_t w, uint32_t (&a)[4]) {
  const uint32_t w8 = w >> 8;
  a[0] = w & 0x000F000Fu;
  a[1] = w & 0x00F000F0u;
  a[2] = w8 & 0x000F000Fu;
  a[3] = w8 & 0x00F000F0u;
}

// The same word decoded to fp16 A fragments with no conversion-unit work: masking
// nibbles into the mantissa of fp16 1024.0 (0x6400) gives 1024 + u (nibbles 0, 2 of
// each half) or 1024 + 16u (nibbles 1, 3, left in place), then one HADD2 / HFMA2
// leaves q exactly.  Register j again holds nibbles (j, j + 4).
__device__ __forceinline__ void dequant_w4_word_f16(uint32_t w, uint32_t (&a)[4]) {
  const uint32_t LO = 0x000F000Fu, HI = 0x00F000F0u, EXP = 0x64006400u;
  const uint32_t w8 = w >> 8;
  uint32_t r[4] = {lop3_and_or(w, LO, EXP), lop3_and_or(w, HI, EXP), lop3_and_or(w8, LO, EXP),
                   lop3_and_or(w8, HI, EXP)};
  const __half2 sub_lo = __halves2half2(__ushort_as_half(0xE408u), __ushort_as_half(0xE408u));   // -1032
  const __half2 mul_hi = __halves2half2(__ushort_as_half(0x2C00u), __ushort_as_half(0x2C00u));   // 1/16
  const __half2 sub_hi = __halves2half2(__ushort_as_half(0xD480u), __ushort_as_half(0xD480u));   // -72
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __half2 v = *reinterpret_cast<__half2*>(&r[j]);
    v = (j & 1) ? __hfma2(v, mul_hi, sub_hi) : __hadd2(v, sub_lo);
    a[j] = *reinterpret_cast<uint32_t*>(&v);
  }
}

// bf16 -> fp16 of 8 packed values (exact for |x| in [2^-14, 65504]; saturates beyond).
__device__ __forceinline__ uint4 bf16x8_to_f16x8(uint4 u) {
  uint32_t in[4] = {u.x, u.y, u.z, u.w}, out[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = fminf(fmaxf(__uint_as_float(in[i] << 16), -65504.f), 65504.f);
    const float hi = fminf(fmaxf(__uint_as_float(in[i] & 0xFFFF0000u), -65504.f), 65504.f);
    const __half2 h = __floats2half2_rn(lo, hi);
    out[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

__device__ __forceinline__ float2 bf162_to_f2(uint32_t u) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(v);
}

// Orderable 32-bit key of a float (larger float -> larger unsigned key).
__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

}  // namespace qw
