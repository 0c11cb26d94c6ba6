// Streaming linear y = x . W^T for the verify block's tokens (W4A16 or bf16 weights).
// Replaces the quantised / dense projections of fused/model.py:197-204 and
// fused/quantization.py:154-165.  HBM-bound: each weight byte is read once per
// 32-token pass; the CTA splits K across its warps and reduces in shared memory, so
// the result is deterministic and the epilogue can fuse the residual add.
#include <mutex>
#include <utility>
#include <vector>

#include <cooperative_groups.h>

#include "bulk_ring.cuh"
#include "stream_gemm.cuh"

namespace qw {

namespace cg = cooperative_groups;

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
// -0 and +0 get one key, so a -0 logit ties with a +0 one and the lower index wins
// (the stable top-1 rule, targets/cpro/ops/draft-top1/src/reference/top1_cpu.cpp:12-16).
__device__ __forceinline__ unsigned long long argmax_key(float v, int n) {
  const float r = rbf(v);
  return (static_cast<unsigned long long>(float_key(r == 0.f ? 0.f : r)) << 32) |
         (0xFFFFFFFFu - static_cast<uint32_t>(n));
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

// ------------------------------------------------------------------ cluster linear
// Verify-block form (T <= 16 tokens).  Clusters of CL_SIZE CTAs split K: CTA rank r
// owns the K chunks [r * nch / CL_SIZE, (r + 1) * nch / CL_SIZE) of every row tile the
// cluster handles (row tile t goes to cluster t mod clusters), so it stages only its
// slice of the activations.  Its warps take whole tiles of the slice (tile i to warp
// i mod CL_WARPS) and stream them from HBM through per-warp rings of bulk copies, all
// requested before the PDL wait.  Partials meet through distributed shared memory: each
// CTA stores its partial of tile i into the shared memory of rank i mod CL_SIZE, which
// adds the CL_SIZE partials of its tiles in rank order after one cluster barrier: the
// order (and partition) of the streaming kernel's K split with rt = 1, so every output
// has the streaming kernel's bits.
constexpr int CL_SIZE = 8;
constexpr int CL_WARPS = 16;
constexpr int CL_MAXT = 16;
constexpr int CL_PAD = 32;      // 16-bit elements of row padding (conflict-free fragment loads)
constexpr int CL_MAXS = 8;      // ring stages per warp, at most

__device__ int32_t g_linear_wait_status;   // sticky: a bounded wait in a cluster linear expired

static std::mutex g_lin_status_mu;
static int32_t* g_lin_status_ptr[64] = {};

int linear_wait_status_addr(int32_t** out) {
  return symbol_addr_cached(g_linear_wait_status, g_lin_status_ptr, 64, g_lin_status_mu, out,
                            "linear wait status address");
}

struct ClArgs {
  const __nv_bfloat16* x;
  const uint8_t* w;
  void* y;
  int64_t ldy;
  int tokens, n, k, mode;
  int tpc;        // row tiles per cluster, at most (partials buffer)
  int nst;        // ring stages per warp
  long long limit;
  unsigned tx_excess;   // 0 except under qw_debug_inject_wait_timeout
};

__host__ __device__ inline size_t cl_head_bytes(int tpc) {
  const size_t owned = (tpc + CL_SIZE - 1) / CL_SIZE;   // tiles a CTA finishes, at most
  return CL_WARPS * CL_MAXS * 8 + owned * CL_SIZE * 32 * 8 * sizeof(float);
}

template <class Fmt>
__global__ void __launch_bounds__(CL_WARPS * 32, 1) cluster_linear_kernel(ClArgs a) {
  using OT = typename Fmt::OT;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int cid = blockIdx.x / CL_SIZE, ncl = gridDim.x / CL_SIZE;
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = a.k, T = a.tokens;
  const int nch = K / Fmt::KCHUNK;
  const int c0 = rank * nch / CL_SIZE, c1 = (rank + 1) * nch / CL_SIZE, ncs = c1 - c0;
  const int maxc = (nch + CL_SIZE - 1) / CL_SIZE;
  const uint32_t sbytes = maxc * Fmt::CHB, wbytes = ncs * Fmt::CHB;
  const int ntiles = a.n / 16;
  const int my_tiles = cid < ntiles ? (ntiles - 1 - cid) / ncl + 1 : 0;
  const int XS = maxc * Fmt::KCHUNK + CL_PAD;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  // partials received for the tiles this CTA finishes: [tpc / CL_SIZE][CL_SIZE][32][8]
  float* part = reinterpret_cast<float*>(smem + CL_WARPS * CL_MAXS * 8);
  OT* xs = reinterpret_cast<OT*>(smem + cl_head_bytes(a.tpc));                     // [T][XS]
  uint8_t* ring = reinterpret_cast<uint8_t*>(xs) + (static_cast<size_t>(T) * XS * 2 + 127) / 128 * 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nst = a.nst;
  uint8_t* wring = ring + static_cast<size_t>(warp) * nst * sbytes;
  uint64_t* wbar = bars + warp * CL_MAXS;
  const int my_w = warp < my_tiles ? (my_tiles - 1 - warp) / CL_WARPS + 1 : 0;   // tiles of this warp
  if (lane == 0)
    for (int i = 0; i < nst; ++i) mbar_init(wbar + i, 1);
  fence_barrier_init();
  __syncthreads();
  auto src = [&](int j) {
    const int t = cid + (warp + j * CL_WARPS) * ncl;
    return a.w + Fmt::tile_offset(t, K, 0) + static_cast<int64_t>(c0) * Fmt::CHB;
  };
  auto issue = [&](int j) {
    uint64_t* b = wbar + (j % nst);
    fence_proxy_async();
    mbar_arrive_expect_tx(b, wbytes + a.tx_excess);
    bulk_g2s(wring + (j % nst) * sbytes, src(j), wbytes, b);
  };
  if (lane == 0 && wbytes)
    for (int j = 0; j < nst && j < my_w; ++j) issue(j);   // weights: before the wait
  pdl_wait();
  pdl_trigger();
  // this CTA's slice of the activations
  const int xw = ncs * Fmt::KCHUNK;
  for (int i = threadIdx.x; i < T * (xw / 8); i += blockDim.x) {
    const int r = i / (xw / 8), c = (i % (xw / 8)) * 8;
    cp_async16(xs + r * XS + c, a.x + static_cast<int64_t>(r) * K + c0 * Fmt::KCHUNK + c, true);
  }
  cp_async_commit();
  cp_async_wait<0>();
  if constexpr (!std::is_same<OT, __nv_bfloat16>::value) {
    // fp16 operands: convert the slice once (each thread the vectors it copied)
    for (int i = threadIdx.x; i < T * (xw / 8); i += blockDim.x) {
      uint4* p = reinterpret_cast<uint4*>(xs + (i / (xw / 8)) * XS + (i % (xw / 8)) * 8);
      *p = bf16x8_to_f16x8(*p);
    }
  }
  __syncthreads();
  const int gid = lane >> 2;
  const bool two = T > 8;
  const OT* xr[2];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) xr[nt] = xs + min(nt * 8 + gid, T - 1) * XS;
  bool ok = true;
  for (int j = 0; j < my_w; ++j) {
    float acc[2][4];
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) acc[jj][0] = acc[jj][1] = acc[jj][2] = acc[jj][3] = 0.f;
    if (wbytes && ok) {
      if (!mbar_wait(wbar + (j % nst), static_cast<uint32_t>((j / nst) & 1), &g_linear_wait_status, a.limit)) {
        if (lane == 0) {   // wait (bounded) for this warp's other copies in flight before giving up
          for (int q = j + 1; q < min(j + nst, my_w); ++q) {
            const long long t0 = clock64();
            while (!mbar_try_wait(wbar + (q % nst), static_cast<uint32_t>((q / nst) & 1)))
              if (clock64() - t0 > a.limit) break;
          }
        }
        ok = false;
      }
      if (ok) {
        const uint8_t* st = wring + (j % nst) * sbytes;
        if constexpr (Fmt::SCALED) {
          if (two) {
            for (int c = 0; c < ncs; ++c) w4_smem_chunks<Fmt::KCHUNK, 1, 2, OT>(st + c * Fmt::CHB, xr, c * Fmt::KCHUNK, lane, acc);
          } else {
            for (int c = 0; c < ncs; ++c) w4_smem_chunks<Fmt::KCHUNK, 1, 1, OT>(st + c * Fmt::CHB, xr, c * Fmt::KCHUNK, lane, acc);
          }
        } else {
          for (int c = 0; c < ncs; ++c) {
            if (two) b16_smem_chunk<2>(st + c * Fmt::CHB, xr, c * Fmt::KCHUNK, lane, acc);
            else b16_smem_chunk<1>(st + c * Fmt::CHB, xr, c * Fmt::KCHUNK, lane, acc);
          }
        }
        __syncwarp();
        if (lane == 0 && j + nst < my_w) issue(j + nst);
      }
    }
    // push the partial to the owner of tile i (rank i mod CL_SIZE), into its slot for
    // this rank: remote stores, no round trip
    const int i = warp + j * CL_WARPS;
    float* dst = cluster.map_shared_rank(part, i % CL_SIZE) +
                 ((static_cast<size_t>(i / CL_SIZE) * CL_SIZE + rank) * 32 + lane) * 8;
    reinterpret_cast<float4*>(dst)[0] = make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
    reinterpret_cast<float4*>(dst)[1] = make_float4(acc[1][0], acc[1][1], acc[1][2], acc[1][3]);
  }
  cluster.sync();   // every partial has reached its owner
  {
    // 256 threads per owned tile (fragment lane l, value e); CL_WARPS / 8 tiles at a time
    const int l = (threadIdx.x & 255) >> 3, e = threadIdx.x & 7;
    const int jj = e >> 2, r = e & 3;
    const int t = jj * 8 + 2 * (l & 3) + (r & 1);
    const int row = (l >> 2) + 8 * (r >> 1);
    for (int i = rank + CL_SIZE * (threadIdx.x >> 8); i < my_tiles; i += CL_SIZE * (CL_WARPS / 8)) {
      float v = 0.f;
#pragma unroll
      for (int sr = 0; sr < CL_SIZE; ++sr)
        v += part[((static_cast<size_t>(i / CL_SIZE) * CL_SIZE + sr) * 32 + l) * 8 + e];
      if (t < T) {
        const int64_t o = static_cast<int64_t>(t) * a.ldy + (cid + i * ncl) * 16 + row;
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

static int cl_sm_count() {
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

struct ClPlan {
  int ncl, tpc, nst;
  size_t smem;
};

template <class Fmt>
static bool cl_plan(const LinArgs& l, int ncl, ClPlan& p) {
  constexpr size_t LIMIT = 227 * 1024;
  const int ntiles = l.n / 16;
  p.ncl = ncl;
  p.tpc = (ntiles + ncl - 1) / ncl;
  const int nch = l.k / Fmt::KCHUNK;
  const int maxc = (nch + CL_SIZE - 1) / CL_SIZE;
  const size_t sbytes = static_cast<size_t>(maxc) * Fmt::CHB;
  const size_t fixed = cl_head_bytes(p.tpc) +
                       (static_cast<size_t>(l.tokens) * (maxc * Fmt::KCHUNK + CL_PAD) * 2 + 127) / 128 * 128;
  const int tpw = (p.tpc + CL_WARPS - 1) / CL_WARPS;   // tiles per warp, at most
  p.nst = tpw < CL_MAXS ? tpw : CL_MAXS;
  while (p.nst > 1 && fixed + CL_WARPS * p.nst * sbytes > LIMIT) --p.nst;
  p.smem = fixed + CL_WARPS * p.nst * sbytes;
  return p.smem <= LIMIT;
}

// Clusters of this kernel and shared-memory size that can be resident at once (8-CTA
// clusters must fit in one GPC); cached per (device, kernel, size).
template <class Fmt>
static int cl_resident(size_t smem) {
  static std::mutex mu;
  static std::vector<std::pair<long long, int>> cache;
  int dev = 0;
  (void)cudaGetDevice(&dev);
  const long long key = (static_cast<long long>(dev) << 40) | static_cast<long long>(smem);
  std::lock_guard<std::mutex> guard(mu);
  for (const auto& kv : cache)
    if (kv.first == key) return kv.second;
  cudaLaunchConfig_t occ = {};
  occ.gridDim = dim3(CL_SIZE);
  occ.blockDim = dim3(CL_WARPS * 32);
  occ.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL_SIZE;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  occ.attrs = attr;
  occ.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, cluster_linear_kernel<Fmt>, &occ) != cudaSuccess || n <= 0) {
    (void)cudaGetLastError();
    n = cl_sm_count() / CL_SIZE;
  }
  cache.emplace_back(key, n);
  return n;
}

// The cluster linear when the block fits (T <= 16, aligned activations); otherwise
// QW_ERR_UNSUPPORTED, and the caller streams.
template <class Fmt>
static int launch_linear_cluster(const LinArgs& l, cudaStream_t s) {
  constexpr size_t LIMIT = 227 * 1024;
  if (l.tokens < 1 || l.tokens > CL_MAXT || l.k % (8 * CL_SIZE) || (reinterpret_cast<uintptr_t>(l.x) & 15))
    return QW_ERR_UNSUPPORTED;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    err = cudaFuncSetAttribute(cluster_linear_kernel<Fmt>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(LIMIT));
  });
  if (err != cudaSuccess) return cuda_status(err, "cluster linear smem attribute");
  const int ntiles = l.n / 16;
  int ncl = cl_sm_count() / CL_SIZE;
  if (ncl > ntiles) ncl = ntiles;
  if (ncl < 1) return QW_ERR_UNSUPPORTED;
  ClPlan p{};
  if (!cl_plan<Fmt>(l, ncl, p)) return QW_ERR_UNSUPPORTED;
  // no second wave of clusters: shrink to the resident count (more tiles per cluster)
  for (int it = 0; it < 3; ++it) {
    const int res = cl_resident<Fmt>(p.smem);
    if (res >= p.ncl) break;
    if (!cl_plan<Fmt>(l, res, p)) return QW_ERR_UNSUPPORTED;
  }
  const WaitInjection inj = wait_injection();
  ClArgs a{l.x, l.w, l.y, l.ldy, l.tokens, l.n, l.k, l.mode, p.tpc, p.nst,
           inj.limit > 0 ? inj.limit : QW_WAIT_LIMIT, inj.tx_excess};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.ncl * CL_SIZE);
  cfg.blockDim = dim3(CL_WARPS * 32);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL_SIZE;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, cluster_linear_kernel<Fmt>, a);
  if (e != cudaSuccess) return cuda_status(e, "linear (cluster)");
  return QW_OK;
}

// One row tile per CTA, K split over its SG_WARPS warps: the partition (and the order
// in which the partial sums are added) of the cluster kernel, so a token's output has
// the same bits whichever kernel (block size) computes it.
static int choose_rt(int /*ntiles*/) { return 1; }

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
  static_assert(SG_WARPS == CL_SIZE, "the streaming and cluster kernels share the 8-way K partition");
  const int rc = launch_linear_cluster<Fmt>(a, s);
  if (rc != QW_ERR_UNSUPPORTED) return rc;
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
    // fp16 MMA operands: the int4 decode then needs no conversion-unit work
    case 128: return dispatch_nt<W4Fmt<128, __half>, 4>(a, s);
    case 64: return dispatch_nt<W4Fmt<64, __half>, 4>(a, s);
    default: return dispatch_nt<W4Fmt<32, __half>, 4>(a, s);
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
