// Small-batch GEMV (M = 1..16): linear_decode, and the MLP gate/up stage on
// its own.  One launch streams one weight through the TMA ring of
// fd_stream.cuh (stream-K over 128-row blocks, two producer warps, eight
// mma.sync / FMA consumer warps, deterministic split-K).  Launches use
// programmatic dependent launch: the weight prefetch is issued before
// griddepcontrol.wait, so it overlaps the previous kernel's tail.
#include "fd_stream.cuh"

#include <map>
#include <mutex>
#include <tuple>

using namespace fd;
using namespace fd_stream;

namespace {

// One phase per launch.  KIND 0 = dot (mma.sync), 1 = simt.  MP = padded
// batch for simt (1..16).  NT = 8-wide MMA batch tiles (1 for m <= 8, 2 for
// m <= 16).  MAXT / MINB: launch bounds (threads, resident CTAs per SM).
template <typename T, int NT, int KIND, int MP, int MODE, int MAXT, int MINB>
__global__ void __launch_bounds__(MAXT, MINB)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                    const GemvArgs a) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ int s_last;
  __shared__ int s_abort;
  __shared__ float s_sumsq[GW][MT_MAX];
  __shared__ __align__(8) uint64_t s_mid[2];
  __shared__ __align__(8) uint64_t s_nw_bar;  // norm weight copy landed (GATEUP)
  __shared__ int s_mid_last, s_fast, s_decided;
  const int nes = a.norm_dtype == FD_F32 ? 4 : 2;
  const int64_t xbytes = MODE == MODE_GATEUP ? static_cast<int64_t>(gateup_region_bytes(a.m, a.ks, a.boxes, a.k, nes))
                                             : static_cast<int64_t>(a.stages) * a.boxes * a.x_slot;
  const Ring r = carve_ring(smem_raw, a.stages, a.boxes, a.x_slot, xbytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = static_cast<int>(blockDim.x >> 5) - GW - 1;  // warps: consumers, producers, announcer
  const int64_t G = gridDim.x, c = blockIdx.x;
  const int64_t s0 = range_start(c, a.total, G);
  const int64_t s1 = range_start(c + 1, a.total, G);
  const MidSync ms{&s_mid[0], &s_mid[1], &s_mid_last, &s_fast, &s_decided, 0u, 1};
  unsigned char* nw_smem = r.xreg + gateup_x_bytes(a.m, a.ks, a.boxes);  // GATEUP: norm weight copy

  if (threadIdx.x == 0) {
    mbar_init(&s_mid[0], GW);
    mbar_init(&s_mid[1], 1);
    mbar_init(&s_nw_bar, 1);
    ring_init(r);  // ends with the mbarrier-init fence
    s_abort = 0;
    s_fast = 0;
    s_decided = 0;
  }
  __syncthreads();

  if (warp == GW + P) {
    // The split-K counters are shared with the previous launch on this
    // workspace: look at them only once that launch has completed.
    grid_dep_wait();
    if (lane == 0) announce_mid(a, ms, s0, s1, G, &s_abort);
    __syncwarp();
    if (gateup_mode(MODE)) watch_final_staged<NT>(a, ms, s0, s1, G, c, r.fin);
    grid_dep_launch();
    return;
  }

  if (warp >= GW) {
    // producer warps: producer p issues ring indices p, p+P, ...
    const int p = warp - GW;
    if (lane == 0) {
      if (MODE == MODE_GATEUP && p == 0) {
        // the norm weight is an input, not the previous kernel's output: copy it now
        const uint32_t nb = static_cast<uint32_t>(a.k * nes);
        mbar_expect_tx(&s_nw_bar, nb);
        bulk_load(nw_smem, a.norm_w, nb, &s_nw_bar);
      }
      prefetch_map(&wmap);
      if (streams_x(MODE)) prefetch_map(&xmap);
      produce_phase<MODE>(r, &wmap, &xmap, a, s0, s1, 0, p, P, evict_first_policy(), &s_abort, [] {
        grid_dep_wait();  // the activation is the previous kernel's output
        return true;
      });
      producer_drain(r, s1 - s0, p, P);
    }
    grid_dep_launch();
    return;
  }
  // consumer warps
  grid_dep_wait();
  if (MODE == MODE_GATEUP) norm_to_smem<T>(a, a.hidden, r, s_sumsq, nw_smem, &s_nw_bar);
  grid_dep_launch();
  consume_phase<T, NT, KIND, MP, MODE>(a, r, s0, s1, 0, G, c, &s_last, &s_abort, ms);
}

// The gate/up stage's RMSNorm on its own, for the streamed gate/up mode: one
// CTA of CONSUMERS threads per row writes normed[row] = round((x * scale) *
// w) with norm_rows's arithmetic -- thread t sums the squares of vectors t,
// t + CONSUMERS, ... as f32x2 pairs, then each warp, then the warps in
// order; the same products -- so the bits equal the resident mode's
// normalised batch.
template <typename T>
__global__ void __launch_bounds__(CONSUMERS) norm_rows_kernel(const GemvArgs a, T* __restrict__ normed) {
  __shared__ float s_part[GW];
  __shared__ float s_scale;
  constexpr int VW = 4;  // vectors of a thread in flight (all of them for k <= 8192)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t row = blockIdx.x;
  const int nvec = static_cast<int>(a.k / 8);
  grid_dep_wait();  // hidden is the previous kernel's output
  grid_dep_launch();
  const uint4* x = reinterpret_cast<const uint4*>(static_cast<const T*>(a.hidden) + row * a.hidden_stride);
  uint4 raw[VW];
  uint64_t acc = 0;  // {+0.f, +0.f}
  for (int v0 = tid; v0 < nvec; v0 += VW * CONSUMERS) {
#pragma unroll
    for (int u = 0; u < VW; ++u) {
      const int v = v0 + u * CONSUMERS;
      raw[u] = v < nvec ? __ldcg(x + v) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < VW; ++u) {
      if (v0 + u * CONSUMERS >= nvec) break;
      const uint64_t p0 = pair_f32x2<T>(raw[u].x), p1 = pair_f32x2<T>(raw[u].y);
      const uint64_t p2 = pair_f32x2<T>(raw[u].z), p3 = pair_f32x2<T>(raw[u].w);
      acc = fma_f32x2(p0, p0, acc);
      acc = fma_f32x2(p1, p1, acc);
      acc = fma_f32x2(p2, p2, acc);
      acc = fma_f32x2(p3, p3, acc);
    }
  }
  const float2 hs = f32x2_split(acc);
  const float t = warp_sum(hs.x + hs.y);
  if (lane == 0) s_part[warp] = t;
  __syncthreads();
  if (tid == 0) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < GW; ++w) tot += s_part[w];
    s_scale = rsqrtf(tot / static_cast<float>(a.k) + a.eps);
  }
  __syncthreads();
  const uint64_t i2 = f32x2_of(s_scale, s_scale);
  const int wes = a.norm_dtype == FD_F32 ? 4 : 2;
  const unsigned char* nw = static_cast<const unsigned char*>(a.norm_w);
  uint4* y = reinterpret_cast<uint4*>(normed + row * a.k);
  const bool kept = nvec <= VW * CONSUMERS;  // every vector of this thread is still in raw[]
#pragma unroll 1
  for (int u = 0, v = tid; v < nvec; ++u, v += CONSUMERS) {
    uint4 xv;
    if (kept) {
#pragma unroll
      for (int uu = 0; uu < VW; ++uu)
        if (uu == u) xv = raw[uu];
    } else {
      xv = __ldcg(x + v);
    }
    uint64_t w[4];
    nw_pairs(nw + static_cast<int64_t>(v) * 8 * wes, a.norm_dtype, w);
    const float2 o0 = f32x2_split(mul_f32x2(mul_f32x2(pair_f32x2<T>(xv.x), i2), w[0]));
    const float2 o1 = f32x2_split(mul_f32x2(mul_f32x2(pair_f32x2<T>(xv.y), i2), w[1]));
    const float2 o2 = f32x2_split(mul_f32x2(mul_f32x2(pair_f32x2<T>(xv.z), i2), w[2]));
    const float2 o3 = f32x2_split(mul_f32x2(mul_f32x2(pair_f32x2<T>(xv.w), i2), w[3]));
    uint4 packed;
    packed.x = pack2<T>(o0.x, o0.y);
    packed.y = pack2<T>(o1.x, o1.y);
    packed.z = pack2<T>(o2.x, o2.y);
    packed.w = pack2<T>(o3.x, o3.y);
    y[v] = packed;
  }
}

// ------------------------------------------------------------ cluster split
// LINEAR GEMV for shapes whose 128-row blocks number about the SMs / S
// (the MLP's down projection: 32 blocks): a thread-block cluster of S = 2 or
// 4 CTAs takes one block, CTA r streaming K steps [r*ks/S, (r+1)*ks/S) of
// it.  Every CTA moves the same bytes, no block is shared across clusters,
// and the split-K sum goes through distributed shared memory: each other
// CTA sends its partial into the cluster leader's shared memory with
// st.async, counted in bytes on an mbarrier there, and exits; the leader
// waits on that mbarrier alone, adds the S partials in rank order
// (deterministic) and runs the epilogue -- no global slots, fences,
// counters, atomics or cluster barrier at the end.  Only the local GPU's
// shared memory is touched; nothing uses TMA multicast.
constexpr int kClusterProducers = 2;
constexpr int kClusterThreads = CONSUMERS + 32 * kClusterProducers;
constexpr int kClusterMaxSplit = 4;

// Partial rows in the leader are padded from MT_MAX to 20 floats: a warp's
// float2 reads of rows 16w + g (g = 0..7) then touch each bank at most twice.
constexpr int kPartStride = 20;
__host__ __device__ inline size_t cluster_part_bytes(int split) {
  return static_cast<size_t>(split - 1) * BR * kPartStride * sizeof(float);
}

template <typename T, int NT, int KIND, int MP, int MODE>
__global__ void __launch_bounds__(kClusterThreads, 1)
    gemv_cluster_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                        const GemvArgs a) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ int s_last, s_abort;
  __shared__ __align__(8) uint64_t s_mid[2];
  __shared__ __align__(8) uint64_t s_part_full;  // leader: the other CTAs' partials have landed
  __shared__ int s_mid_last, s_fast, s_decided;
  const int64_t xb = static_cast<int64_t>(a.stages) * a.boxes * a.x_slot;
  const Ring r = carve_ring(smem_raw, a.stages, a.boxes, a.x_slot, xb + cluster_part_bytes(a.cl_split));
  float* part = reinterpret_cast<float*>(r.xreg + xb);  // [split - 1][BR][kPartStride]: in the leader
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const uint32_t rank = cluster_ctarank();
  const int split = a.cl_split;
  const int64_t blk = blockIdx.x / split;
  const int64_t s0 = blk * a.ks + rank * a.ks / split, s1 = blk * a.ks + (rank + 1) * a.ks / split;
  const MidSync ms{&s_mid[0], &s_mid[1], &s_mid_last, &s_fast, &s_decided, 0u, 1};  // no mid blocks here
  if (threadIdx.x == 0) {
    mbar_init(&s_part_full, 1);
    ring_init(r);  // ends with the mbarrier-init fence (cluster scope)
    s_abort = 0;
    // the leader expects 16 * NT bytes from every consumer thread of the other CTAs
    if (rank == 0) mbar_expect_tx(&s_part_full, static_cast<uint32_t>((split - 1) * CONSUMERS * NT * 16));
  }
  __syncthreads();
  cluster_arrive_relaxed();  // phase 1: this CTA (and its shared memory) is running

  Acc<NT> acc, ex;
  acc.zero();
  ex.zero();
  if (warp >= GW) {
    const int p = warp - GW;
    if (lane == 0 && p < a.cl_producers) {  // the other producer warp, if any, idles
      prefetch_map(&wmap);
      prefetch_map(&xmap);
      produce_phase<MODE_LINEAR>(r, &wmap, &xmap, a, s0, s1, 0, p, a.cl_producers, evict_first_policy(), &s_abort,
                                 [] {
                                   grid_dep_wait();  // the activation is the previous kernel's output
                                   return true;
                                 });
      producer_drain(r, s1 - s0, p, a.cl_producers);
    }
    __syncwarp();
    grid_dep_launch();
  } else {
    grid_dep_wait();
    // The leader's epilogue terms (bias, residual rows) are inputs: load them
    // now, so their L2 round trip overlaps the weight stream instead of
    // following the partials' arrival at the end.
    if (rank == 0) Epilogue<T, NT, MODE>::extras(a, blk, ex);
    grid_dep_launch();
    // Phase 1 complete (every CTA of the cluster is running): waited here,
    // where the first stage's latency hides it, not after the stream.
    cluster_wait();
    consume_phase<T, NT, KIND, MP, MODE>(a, r, s0, s1, 0, 1, 0, &s_last, &s_abort, ms, &acc);
  }
  if (warp >= GW) {
    cluster_wait();  // phase 1 (long complete): every thread takes part in each arrive / wait pair
    return;
  }
  if (rank != 0) {
    // The partial goes to the leader with st.async, counted on its mbarrier:
    // no fence and no second cluster barrier, and this CTA is done.
    const uint32_t bar = cluster_map(&s_part_full, 0);
    float* slot = part + (rank - 1) * (BR * kPartStride);
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = 16 * warp + g + 8 * h, col = 8 * t + 2 * q;
        st_async_f2(cluster_map(slot + row * kPartStride + col, 0), acc.v[t][2 * h], acc.v[t][2 * h + 1], bar);
      }
    return;
  }
  if (!mbar_wait_cluster(&s_part_full, 0)) {
    atomicOr(a.status, kStatusFullTimeout);
    return;
  }
  // rank order: 0 + (the leader's own partial, from registers) + rank 1 + ...
  Acc<NT> sum;
  sum.zero();
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) sum.v[t][e] += acc.v[t][e];
#pragma unroll 3
  for (int k = 1; k < split; ++k) {
    const float* pk = part + (k - 1) * (BR * kPartStride);
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = 16 * warp + g + 8 * h, col = 8 * t + 2 * q;
        const float2 v = *reinterpret_cast<const float2*>(pk + row * kPartStride + col);
        sum.v[t][2 * h] += v.x;
        sum.v[t][2 * h + 1] += v.y;
      }
  }
  Epilogue<T, NT, MODE>::run(a, blk, sum, ex, r.xchg);
}

// ------------------------------------------------------------ generic GEMV
// Any strides, any K: one warp per output row.  Used for layouts the TMA
// kernel cannot address (transposed weights, unaligned rows, ...).
struct GenArgs {
  const void* x;
  int64_t sxm, sxk;
  const void* w;
  int64_t swn, swk;
  const void* bias;
  int32_t bias_dtype;
  int64_t sbias;
  const void* ra;
  int32_t ra_dtype;
  int64_t srm, srn;
  void* y;
  int64_t sym, syn;
  int32_t m;
  int64_t n, k;
};

template <typename T>
__global__ void __launch_bounds__(256) gemv_generic_kernel(const GenArgs a) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= a.n) return;
  const T* w = static_cast<const T*>(a.w) + row * a.swn;
  const T* x = static_cast<const T*>(a.x);
  float acc[MT_MAX];
#pragma unroll
  for (int mm = 0; mm < MT_MAX; ++mm) acc[mm] = 0.f;
  for (int64_t kk = lane; kk < a.k; kk += 32) {
    const float wv = to_f32(w[kk * a.swk]);
#pragma unroll
    for (int mm = 0; mm < MT_MAX; ++mm)
      if (mm < a.m) acc[mm] = fmaf(wv, to_f32(x[mm * a.sxm + kk * a.sxk]), acc[mm]);
  }
#pragma unroll
  for (int mm = 0; mm < MT_MAX; ++mm) acc[mm] = warp_sum(acc[mm]);
  if (lane == 0) {
    const float bias = a.bias ? load_as_f32(a.bias, a.bias_dtype, row * a.sbias) : 0.f;
#pragma unroll
    for (int mm = 0; mm < MT_MAX; ++mm) {
      if (mm < a.m) {
        float v = acc[mm] + bias;
        if (a.ra) v += load_as_f32(a.ra, a.ra_dtype, mm * a.srm + row * a.srn);
        static_cast<T*>(a.y)[mm * a.sym + row * a.syn] = from_f32<T>(v);
      }
    }
  }
}

// ------------------------------------------------------------ host side
template <typename Kern>
cudaError_t launch_tma(Kern kern, const CUtensorMap& wm, const CUtensorMap& xm, const GemvArgs& a,
                       const Geometry& geo, size_t smem, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(fd_host::sm_count(), a.total));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(CONSUMERS + 32 * (geo.producers + 1));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, wm, xm, a);
}

template <typename T, int MODE>
cudaError_t dispatch_tma(const CUtensorMap& wm, const CUtensorMap& xm, const GemvArgs& a, int kind,
                         const Geometry& geo, size_t smem, cudaStream_t st) {
  auto L = [&](auto kern) { return launch_tma(kern, wm, xm, a, geo, smem, st); };
  constexpr int MT1 = CONSUMERS + 32 * (MAX_PRODUCERS + 1);
  if (kind == FD_KIND_DOT) {
    if (a.m <= 8) return L(gemv_tma_kernel<T, 1, 0, 1, MODE, MT1, 1>);
    return L(gemv_tma_kernel<T, 2, 0, 1, MODE, MT1, 1>);
  }
  if constexpr (MODE == MODE_LINEAR_TP) {
    return cudaErrorInvalidValue;  // dot only (launch_linear)
  } else {
    if (a.m <= 1) return L(gemv_tma_kernel<T, 1, 1, 1, MODE, MT1, 1>);
    if (a.m <= 2) return L(gemv_tma_kernel<T, 1, 1, 2, MODE, MT1, 1>);
    if (a.m <= 4) return L(gemv_tma_kernel<T, 1, 1, 4, MODE, MT1, 1>);
    if (a.m <= 8) return L(gemv_tma_kernel<T, 1, 1, 8, MODE, MT1, 1>);
    return L(gemv_tma_kernel<T, 2, 1, 16, MODE, MT1, 1>);
  }
}

// Cluster size for a LINEAR launch, 0 for stream-K: the largest S in {4, 2}
// with blocks * S between 80 % and 100 % of the SMs and at least S steps per
// block; FD_GEMV_CLUSTER=0 turns the cluster split off (tuning).
int cluster_split(const GemvArgs& a, const Geometry& geo) {
  const char* env = std::getenv("FD_GEMV_CLUSTER");
  if (env && env[0] == '0') return 0;
  const int64_t sms = fd_host::sm_count();
  const size_t limit = kSmemPerCta;
  for (int s = kClusterMaxSplit; s >= 2; s /= 2) {
    const int64_t ctas = a.nblocks * s;
    if (ctas <= sms && ctas * 10 >= sms * 8 && a.ks >= s &&
        ring_smem_bytes(linear_x_bytes(a.m, geo.stages, geo.boxes) + cluster_part_bytes(s), geo.stages,
                        geo.boxes) <= limit)
      return s;
  }
  return 0;
}

template <typename Kern>
cudaError_t launch_cluster(Kern kern, const CUtensorMap& wm, const CUtensorMap& xm, const GemvArgs& a, size_t smem,
                           cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.nblocks * a.cl_split));
  cfg.blockDim = dim3(kClusterThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(a.cl_split);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  // every cluster must be resident at once for the split to pay: else stream-K
  // (the answer depends on the kernel, its shared memory and the cluster size)
  static std::mutex mu;
  static std::map<std::tuple<const void*, size_t, int, int>, int> fits;
  int dev = 0;
  (void)cudaGetDevice(&dev);
  const auto key = std::make_tuple(reinterpret_cast<const void*>(kern), smem, a.cl_split, dev);
  int clusters = -1;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = fits.find(key);
    if (it != fits.end()) clusters = it->second;
  }
  if (clusters < 0) {
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      clusters = 0;
    }
    std::lock_guard<std::mutex> lock(mu);
    fits[key] = clusters;
  }
  if (clusters < a.nblocks) return cudaErrorUnsupportedLimit;
  return cudaLaunchKernelEx(&cfg, kern, wm, xm, a);
}

template <typename T, int MODE>
cudaError_t dispatch_cluster(const CUtensorMap& wm, const CUtensorMap& xm, const GemvArgs& a, int kind, size_t smem,
                             cudaStream_t st) {
  auto L = [&](auto kern) { return launch_cluster(kern, wm, xm, a, smem, st); };
  if (kind == FD_KIND_DOT) {
    if (a.m <= 8) return L(gemv_cluster_kernel<T, 1, 0, 1, MODE>);
    return L(gemv_cluster_kernel<T, 2, 0, 1, MODE>);
  }
  if constexpr (MODE == MODE_LINEAR_TP) {
    return cudaErrorInvalidValue;  // dot only (launch_linear)
  } else {
    if (a.m <= 1) return L(gemv_cluster_kernel<T, 1, 1, 1, MODE>);
    if (a.m <= 2) return L(gemv_cluster_kernel<T, 1, 1, 2, MODE>);
    if (a.m <= 4) return L(gemv_cluster_kernel<T, 1, 1, 4, MODE>);
    if (a.m <= 8) return L(gemv_cluster_kernel<T, 1, 1, 8, MODE>);
    return L(gemv_cluster_kernel<T, 2, 1, 16, MODE>);
  }
}

// Launch the stream-K TMA GEMV in LINEAR mode: y = x @ w^T (+bias)(+row_add).
// tp_fold: the tensor-parallel epilogue that also sums the ranks
// (MODE_LINEAR_TP, kind = dot only).
int launch_linear(const void* x, int64_t sxm, const void* w, int64_t swn, GemvArgs a, int dtype, int kind,
                  const Workspace& ws, cudaStream_t st, bool tp_fold = false) {
  const int m = a.m;
  const Geometry geo = choose_geometry([m](int stages, int boxes) { return linear_x_bytes(m, stages, boxes); });
  if (geo.stages == 0) return FD_ERR_UNSUPPORTED;
  a.boxes = geo.boxes;
  a.stages = geo.stages;
  a.ks = (a.k + static_cast<int64_t>(geo.boxes) * KC - 1) / (static_cast<int64_t>(geo.boxes) * KC);
  a.nblocks = (a.n + BR - 1) / BR;
  if (a.nblocks > kMaxCounters) return FD_ERR_UNSUPPORTED;
  a.total = a.nblocks * a.ks;
  a.x_slot = x_slot_bytes(a.m);
  a.slots = ws.slots; a.counters = ws.counters; a.status = ws.status;
  CUtensorMap wm, xm;
  // A single row's stride is never used by the TMA unit; keep it legal.
  const int64_t xstride = a.m == 1 ? ((a.k + 7) / 8) * 8 : sxm;
  if (!make_map_2d(&wm, w, a.n, a.k, swn, BR) || !make_map_2d(&xm, x, a.m, a.k, xstride, a.m))
    return FD_ERR_LAUNCH;
  // The cluster kernel's ring: 5 stages instead of 4 where each CTA streams
  // at least 16 steps of a batch of up to 8 rows, its 2 producer warps taking
  // alternate ring indices (a stage's refills then alternate between them:
  // each waits for its own index's stage to be released and arms the full
  // barrier only after that).  Measured on B200, same call: down projection
  // at Llama-3-8B widths 20.96 -> 20.54 us (M = 1), 21.21 -> 20.72 (M = 8);
  // at 70B widths 74.7 -> 72.0, 75.1 -> 72.7; the 8B MLP stack 60.9 -> 60.3
  // us/layer at M = 1.  Not taken where it measured slower: 8 steps per CTA
  // (N = K = 4096: +0.1 to +0.3 us) and 16-row batches (the stack +0.3).
  // One producer for 5 stages was 55 % slower.  FD_GEMV_GEOMETRY sets the
  // geometry instead.
  Geometry cgeo = geo;
  cgeo.producers = std::min(geo.producers, kClusterProducers);
  int split = cluster_split(a, cgeo);
  if (split > 1 && a.m <= 8 && a.ks / split >= 16 && !std::getenv("FD_GEMV_GEOMETRY")) {
    const Geometry deep{kClusterProducers, geo.boxes, 5};
    if (ring_smem_bytes(linear_x_bytes(a.m, deep.stages, deep.boxes) + cluster_part_bytes(split), deep.stages,
                        deep.boxes) <= kSmemPerCta)
      cgeo = deep;
  }
  if (split > 1) {
    a.cl_split = split;
    a.cl_producers = cgeo.producers;
    a.stages = cgeo.stages;
    const size_t csmem =
        ring_smem_bytes(linear_x_bytes(a.m, a.stages, a.boxes) + cluster_part_bytes(split), a.stages, a.boxes);
    cudaError_t e = tp_fold ? (dtype == FD_BF16 ? dispatch_cluster<__nv_bfloat16, MODE_LINEAR_TP>(wm, xm, a, kind, csmem, st)
                                                : dispatch_cluster<__half, MODE_LINEAR_TP>(wm, xm, a, kind, csmem, st))
                            : (dtype == FD_BF16 ? dispatch_cluster<__nv_bfloat16, MODE_LINEAR>(wm, xm, a, kind, csmem, st)
                                                : dispatch_cluster<__half, MODE_LINEAR>(wm, xm, a, kind, csmem, st));
    if (e == cudaSuccess) return FD_OK;
    if (e != cudaErrorUnsupportedLimit) return FD_ERR_LAUNCH;
    (void)cudaGetLastError();  // the clusters do not fit the device: stream-K below
    a.cl_split = 0;
    a.stages = geo.stages;
  }
  // Stream-K: 5 stages under the same rule as the cluster kernel's ring
  // (measured on B200, same call: N = 28672 K = 4096 40.4 -> 39.2 us at M = 1,
  // 39.4 -> 38.9 at M = 8; N = 14336 -0.2 to -0.3 us; at M = 16 0.5 us slower).
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(fd_host::sm_count(), a.total));
  if (a.m <= 8 && geo.stages == 4 && geo.producers == 2 && a.total / grid >= 16 && !std::getenv("FD_GEMV_GEOMETRY") &&
      ring_smem_bytes(linear_x_bytes(a.m, 5, a.boxes), 5, a.boxes) <= kSmemPerCta)
    a.stages = 5;
  const size_t smem = ring_smem_bytes(linear_x_bytes(a.m, a.stages, a.boxes), a.stages, a.boxes);
  cudaError_t e = tp_fold ? (dtype == FD_BF16 ? dispatch_tma<__nv_bfloat16, MODE_LINEAR_TP>(wm, xm, a, kind, geo, smem, st)
                                              : dispatch_tma<__half, MODE_LINEAR_TP>(wm, xm, a, kind, geo, smem, st))
                          : (dtype == FD_BF16 ? dispatch_tma<__nv_bfloat16, MODE_LINEAR>(wm, xm, a, kind, geo, smem, st)
                                              : dispatch_tma<__half, MODE_LINEAR>(wm, xm, a, kind, geo, smem, st));
  return from_cuda(e);
}

// RMSNorm (prologue) -> gate/up GEMV -> SwiGLU -> mid [m, i].
// Which gate/up mode a launch takes: the resident normalised batch (GATEUP:
// the RMSNorm in the kernel's prologue) while it leaves the ring its full
// depth; else the streamed batch (norm_rows_kernel, then GATEUP_S streaming
// the normalised rows with the weights) -- one launch more, but a full ring
// (8B widths above 10 rows, 70B widths above 4).  FD_GATEUP_STREAM = 1 / 0
// forces one or the other (tests, tuning).
struct GateUpPlan {
  Geometry geo;
  bool streamed;
};

GateUpPlan plan_gate_up(int m, int64_t h, int nes) {
  Geometry res = choose_geometry([m, h, nes](int, int boxes) {
    const int64_t ks = (h + static_cast<int64_t>(boxes) * KC - 1) / (static_cast<int64_t>(boxes) * KC);
    return gateup_region_bytes(m, ks, boxes, h, nes);
  });
  // The resident mode takes a fifth ring stage (the 2 producer warps then
  // alternate on a stage) where it fits with the final block's staging area
  // beside it: small batches.  Measured on B200 at Llama-3-8B widths, M = 1:
  // the gate/up kernel 39.1 -> 38.4 us, the MLP stack 60.3 -> 59.8 us/layer.
  if (!std::getenv("FD_GEMV_GEOMETRY") && res.stages == 4 && res.producers == 2) {
    const int64_t ks = (h + static_cast<int64_t>(res.boxes) * KC - 1) / (static_cast<int64_t>(res.boxes) * KC);
    if (ring_smem_bytes(gateup_region_bytes(m, ks, res.boxes, h, nes), 5, res.boxes) + fin_stage_bytes(1) <=
        kSmemPerCta)
      res.stages = 5;
  }
  const Geometry str = choose_geometry([m](int stages, int boxes) { return linear_x_bytes(m, stages, boxes); });
  const char* env = std::getenv("FD_GATEUP_STREAM");
  if (env && env[0] == '1' && str.stages > 0) return {str, true};
  if (env && env[0] == '0') return {res, false};
  const Geometry full = choose_geometry([](int, int) { return size_t{0}; });  // the ring with no X region
  if (res.stages >= full.stages || str.stages <= res.stages) return {res, false};
  return {str, true};
}

}  // namespace

namespace fd_host {
int mlp_layer_launches(int32_t m, int64_t h, int64_t i, int32_t norm_dtype, int32_t kind, bool tensor_parallel) {
  (void)i;
  int n = plan_gate_up(m, h, norm_dtype == FD_F32 ? 4 : 2).streamed ? 3 : 2;
  if (tensor_parallel && !(kind == FD_KIND_DOT && tp_fold_enabled())) ++n;
  return n;
}
}  // namespace fd_host

namespace {

// MLP workspace tail: mid [m, i], two ping-pong hidden buffers [m, h], then
// the streamed gate/up mode's normalised rows [m, h].
char* normed_rows(const Workspace& ws, int m, int64_t h, int64_t i) {
  const size_t mm = static_cast<size_t>(std::max(m, 1));
  return ws.tail + align256(mm * i * 2) + 2 * align256(mm * h * 2);
}

int launch_gate_up(const void* hidden, const void* norm_w, int32_t norm_dtype, const void* w_gate_up,
                   int64_t s_gu, void* mid, int32_t dtype, int32_t m, int64_t h, int64_t i, float eps, int32_t kind,
                   const Workspace& ws, cudaStream_t st) {
  const int nes = norm_dtype == FD_F32 ? 4 : 2;
  const GateUpPlan plan = plan_gate_up(m, h, nes);
  const Geometry geo = plan.geo;
  if (geo.stages == 0) return FD_ERR_UNSUPPORTED;
  GemvArgs a = {};
  a.y = static_cast<char*>(mid); a.sym = i; a.syn = 1;
  a.m = m; a.n = 2 * i; a.k = h;
  a.boxes = geo.boxes;
  a.stages = geo.stages;
  a.ks = (h + static_cast<int64_t>(geo.boxes) * KC - 1) / (static_cast<int64_t>(geo.boxes) * KC);
  a.nblocks = (i + BR / 2 - 1) / (BR / 2);
  if (a.nblocks > kMaxCounters) return FD_ERR_UNSUPPORTED;
  a.total = a.nblocks * a.ks;
  a.slots = ws.slots; a.counters = ws.counters; a.status = ws.status;
  a.inner = i;
  a.hidden = hidden; a.hidden_stride = h;
  a.norm_w = norm_w; a.norm_dtype = norm_dtype; a.eps = eps;
  CUtensorMap gm, xm;
  if (!make_gate_up_map(&gm, w_gate_up, h, i, s_gu)) return FD_ERR_LAUNCH;
  if (plan.streamed) {
    // the normalised rows first, then [m x 64] boxes of them with each weight step
    char* normed = normed_rows(ws, m, h, i);
    if (!make_map_2d(&xm, normed, m, h, h, m)) return FD_ERR_LAUNCH;
    const cudaError_t en =
        dtype == FD_BF16
            ? fd_host::launch_pdl(norm_rows_kernel<__nv_bfloat16>, dim3(m), CONSUMERS, 0, st, a,
                                  reinterpret_cast<__nv_bfloat16*>(normed))
            : fd_host::launch_pdl(norm_rows_kernel<__half>, dim3(m), CONSUMERS, 0, st, a, reinterpret_cast<__half*>(normed));
    if (en != cudaSuccess) return FD_ERR_LAUNCH;
  }
  a.x_slot = plan.streamed ? x_slot_bytes(m) : 0;
  size_t smem = ring_smem_bytes(plan.streamed ? linear_x_bytes(m, a.stages, a.boxes)
                                              : gateup_region_bytes(m, a.ks, a.boxes, h, nes),
                                a.stages, a.boxes);
  // room for the final block's staged partials (batches up to 8 rows), where
  // it costs no ring stage
  const size_t fin = fin_stage_bytes(1);
  if (m <= 8 && smem + fin <= kSmemPerCta) {
    smem += fin;
    a.fin_stage = 1;
  }
  cudaError_t e;
  if (plan.streamed)
    e = dtype == FD_BF16 ? dispatch_tma<__nv_bfloat16, MODE_GATEUP_S>(gm, xm, a, kind, geo, smem, st)
                         : dispatch_tma<__half, MODE_GATEUP_S>(gm, xm, a, kind, geo, smem, st);
  else
    e = dtype == FD_BF16 ? dispatch_tma<__nv_bfloat16, MODE_GATEUP>(gm, gm, a, kind, geo, smem, st)
                         : dispatch_tma<__half, MODE_GATEUP>(gm, gm, a, kind, geo, smem, st);
  return from_cuda(e);
}

// Argument checks shared by the fused MLP entry points.
int check_mlp_args(const void* hidden, const void* norm_w, int32_t norm_dtype, const void* w_gate_up,
                      int64_t s_gu, int32_t dtype, int32_t m, int64_t h, int64_t i, int32_t kind) {
  using namespace fd_host;
  if (m < 0 || h < 0 || i < 0) return FD_ERR_ARG;
  if (m > MT_MAX) return FD_ERR_UNSUPPORTED;
  if (!hidden || !norm_w || !w_gate_up) return FD_ERR_ARG;
  if (!half_dtype(dtype) || !valid_dtype(norm_dtype)) return FD_ERR_ARG;
  if (kind != FD_KIND_DOT && kind != FD_KIND_SIMT) return FD_ERR_ARG;
  if (h % 8 || i % 8 || i == 0 || s_gu % 8 || s_gu < h) return FD_ERR_UNSUPPORTED;
  if (!aligned16(hidden) || !aligned16(norm_w) || !aligned16(w_gate_up)) return FD_ERR_UNSUPPORTED;
  if ((i + BR / 2 - 1) / (BR / 2) > kMaxCounters || (h + BR - 1) / BR > kMaxCounters) return FD_ERR_UNSUPPORTED;
  if (!encode_fn()) return FD_ERR_DEVICE;
  return FD_OK;
}

// MLP intermediates behind the stream-K workspace: mid [m, i], then two
// ping-pong hidden buffers [m, h] for the layers of a stack, then the
// streamed gate/up mode's normalised rows [m, h] (normed_rows).
size_t mlp_tail_bytes(int m, int64_t h, int64_t i) {
  const size_t mm = static_cast<size_t>(std::max(m, 1));
  return align256(mm * i * 2) + 3 * align256(mm * h * 2);
}

// One post_attn_mlp layer as two launches on `st`: gate/up (RMSNorm prologue,
// SwiGLU epilogue) -> mid, then down (+ residual) -> out.  The second launch
// is programmatic-dependent on the first, so its producers start streaming
// the down weight while the gate/up grid drains.
int mlp_layer(const void* hidden, const void* norm_w, int32_t norm_dtype, const void* w_gate_up, int64_t s_gu,
              const void* w_down, int64_t s_down, void* out, bool out_f32, bool add_residual, int32_t dtype,
              int32_t m, int64_t h, int64_t i, float eps, int32_t kind, const Workspace& ws, cudaStream_t st) {
  char* mid = ws.tail;
  int r = launch_gate_up(hidden, norm_w, norm_dtype, w_gate_up, s_gu, mid, dtype, m, h, i, eps, kind, ws, st);
  if (r != FD_OK) return r;
  GemvArgs b = {};
  b.ra = add_residual ? hidden : nullptr; b.ra_dtype = dtype; b.srm = h; b.srn = 1;
  b.y = static_cast<char*>(out); b.sym = h; b.syn = 1;
  b.y_f32 = out_f32;
  b.m = m; b.n = h; b.k = i;
  return launch_linear(mid, i, w_down, s_down, b, dtype, kind, ws, st);
}

// Checks of the down projection and output shared by the MLP entry points.
int check_down(const void* w_down, int64_t s_down, const void* out, int32_t out_dtype, int32_t dtype, int64_t i) {
  using namespace fd_host;
  if (!w_down || !out) return FD_ERR_ARG;
  if (!(out_dtype == dtype || out_dtype == FD_F32)) return FD_ERR_ARG;
  if (s_down % 8 || s_down < i || !aligned16(w_down)) return FD_ERR_UNSUPPORTED;
  return FD_OK;
}

}  // namespace

extern "C" {

size_t fd_linear_workspace_bytes(int32_t m, int64_t n, int64_t k) {
  (void)m;
  (void)n;
  (void)k;
  return streamk_ws_bytes();
}

size_t fd_workspace_status_offset(void) { return status_offset(); }

int fd_linear_out(const void* x, int64_t sxm, int64_t sxk, const void* w, int64_t swn, int64_t swk,
                  const void* bias, int32_t bias_dtype, int64_t sbias, const void* row_add,
                  int32_t ra_dtype, int64_t srm, int64_t srn, void* y, int64_t sym, int64_t syn,
                  int32_t dtype, int32_t m, int64_t n, int64_t k, int32_t kind, void* workspace,
                  size_t workspace_bytes, void* stream) {
  using namespace fd_host;
  if (m < 0 || n < 0 || k < 0) return FD_ERR_ARG;
  if (m == 0 || n == 0) return FD_OK;
  if (m > MT_MAX) return FD_ERR_UNSUPPORTED;
  if (!x || !w || !y || !half_dtype(dtype)) return FD_ERR_ARG;
  if (kind != FD_KIND_DOT && kind != FD_KIND_SIMT) return FD_ERR_ARG;
  if (bias && !(bias_dtype == dtype || bias_dtype == FD_F32)) return FD_ERR_ARG;
  if (row_add && !valid_dtype(ra_dtype)) return FD_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // The TMA path needs unit k-strides, 16-byte aligned bases and row strides.
  const bool tma = k > 0 && swk == 1 && sxk == 1 && aligned16(x) && aligned16(w) && swn % 8 == 0 &&
                   swn >= k && (m == 1 || (sxm % 8 == 0 && sxm >= k)) && encode_fn() != nullptr;
  if (tma) {
    if (!workspace || workspace_bytes < streamk_ws_bytes()) return FD_ERR_WORKSPACE;
    GemvArgs a = {};
    a.bias = bias; a.bias_dtype = bias_dtype; a.sbias = sbias;
    a.ra = row_add; a.ra_dtype = ra_dtype; a.srm = srm; a.srn = srn;
    a.y = static_cast<char*>(y); a.sym = sym; a.syn = syn;
    a.m = m; a.n = n; a.k = k;
    const int r = launch_linear(x, sxm, w, swn, a, dtype, kind, carve(workspace), st);
    if (r != FD_ERR_UNSUPPORTED) return r;
  }
  GenArgs a;
  a.x = x; a.sxm = sxm; a.sxk = sxk;
  a.w = w; a.swn = swn; a.swk = swk;
  a.bias = bias; a.bias_dtype = bias_dtype; a.sbias = sbias;
  a.ra = row_add; a.ra_dtype = ra_dtype; a.srm = srm; a.srn = srn;
  a.y = y; a.sym = sym; a.syn = syn;
  a.m = m; a.n = n; a.k = k;
  const int64_t threads = n * 32;
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  if (dtype == FD_BF16) gemv_generic_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(a);
  else gemv_generic_kernel<__half><<<blocks, 256, 0, st>>>(a);
  return from_cuda(cudaGetLastError());
}

int fd_mlp_gate_up_out(const void* hidden, const void* norm_w, int32_t norm_dtype, const void* w_gate_up,
                       int64_t s_gu, void* mid, int32_t dtype, int32_t m, int64_t h, int64_t i, float eps,
                       int32_t kind, void* workspace, size_t workspace_bytes, void* stream) {
  const int chk = check_mlp_args(hidden, norm_w, norm_dtype, w_gate_up, s_gu, dtype, m, h, i, kind);
  if (chk != FD_OK) return chk;
  if (m == 0 || h == 0) return FD_OK;
  if (!mid) return FD_ERR_ARG;
  if (!workspace || workspace_bytes < fd_post_attn_mlp_workspace_bytes(m, h, i)) return FD_ERR_WORKSPACE;
  return launch_gate_up(hidden, norm_w, norm_dtype, w_gate_up, s_gu, mid, dtype, m, h, i, eps, kind,
                        carve(workspace), static_cast<cudaStream_t>(stream));
}

size_t fd_post_attn_mlp_workspace_bytes(int32_t m, int64_t h, int64_t i) {
  return streamk_ws_bytes() + mlp_tail_bytes(m, h, i);
}

int fd_post_attn_mlp_out(const void* hidden, const void* norm_w, int32_t norm_dtype, const void* w_gate_up,
                         int64_t s_gu, const void* w_down, int64_t s_down, void* out, int32_t out_dtype,
                         int32_t dtype, int32_t m, int64_t h, int64_t i, float eps, int32_t kind,
                         int32_t add_residual, void* workspace, size_t workspace_bytes, void* stream) {
  int r = check_mlp_args(hidden, norm_w, norm_dtype, w_gate_up, s_gu, dtype, m, h, i, kind);
  if (r != FD_OK) return r;
  if (m == 0 || h == 0) return FD_OK;
  r = check_down(w_down, s_down, out, out_dtype, dtype, i);
  if (r != FD_OK) return r;
  if (!workspace || workspace_bytes < fd_post_attn_mlp_workspace_bytes(m, h, i)) return FD_ERR_WORKSPACE;
  return mlp_layer(hidden, norm_w, norm_dtype, w_gate_up, s_gu, w_down, s_down, out, out_dtype == FD_F32,
                   add_residual != 0, dtype, m, h, i, eps, kind, carve(workspace), static_cast<cudaStream_t>(stream));
}

int fd_post_attn_mlp_tp_out(const void* hidden, const void* norm_w, int32_t norm_dtype, const void* w_gate_up,
                            int64_t s_gu, const void* w_down, int64_t s_down, void* out, int32_t dtype, int32_t m,
                            int64_t h, int64_t i, float eps, int32_t kind, int32_t rank, int32_t world,
                            void* const* exchange, int32_t m_max, void* workspace, size_t workspace_bytes,
                            void* stream) {
  using namespace fd_host;
  int r = check_mlp_args(hidden, norm_w, norm_dtype, w_gate_up, s_gu, dtype, m, h, i, kind);
  if (r != FD_OK) return r;
  if (world < 1 || world > kMaxTpWorld || rank < 0 || rank >= world || !exchange) return FD_ERR_ARG;
  if (m_max < 1 || m_max > MT_MAX || m > m_max) return FD_ERR_ARG;
  for (int k = 0; k < world; ++k)
    if (!exchange[k]) return FD_ERR_ARG;
  if (m == 0 || h == 0) return FD_OK;
  r = check_down(w_down, s_down, out, dtype, dtype, i);
  if (r != FD_OK) return r;
  if (!workspace || workspace_bytes < fd_post_attn_mlp_workspace_bytes(m, h, i)) return FD_ERR_WORKSPACE;
  const Workspace ws = carve(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* mid = ws.tail;
  r = launch_gate_up(hidden, norm_w, norm_dtype, w_gate_up, s_gu, mid, dtype, m, h, i, eps, kind, ws, st);
  if (r != FD_OK) return r;
  // down projection of this rank's shard: block partials go to every rank
  const TpLayout l = tp_layout(world, m_max, h);
  GemvArgs b = {};
  b.m = m; b.n = h; b.k = i;
  for (int k = 0; k < world; ++k) b.tp_peer[k] = static_cast<char*>(exchange[k]);
  b.tp_rank = rank; b.tp_world = world; b.tp_mmax = m_max;
  b.tp_data_off = l.data_off;
  b.tp_seq = static_cast<const int*>(exchange[rank]);
  if (kind == FD_KIND_DOT && tp_fold_enabled()) {
    // opt-in, two launches: each block's finisher also sums the ranks and adds the residual
    b.ra = hidden; b.ra_dtype = dtype; b.srm = h; b.srn = 1;
    b.y = static_cast<char*>(out); b.sym = h; b.syn = 1;
    return launch_linear(mid, i, w_down, s_down, b, dtype, kind, ws, st, true);
  }
  r = launch_linear(mid, i, w_down, s_down, b, dtype, kind, ws, st);
  if (r != FD_OK) return r;
  return tp_reduce_launch(static_cast<char*>(exchange[rank]), world, m, m_max, h, hidden, out, dtype, ws.status, st);
}

int fd_post_attn_mlp_tp_stack_out(const void* hidden, int32_t layers, const void* const* norm_w, int32_t norm_dtype,
                                  const void* const* w_gate_up, int64_t s_gu, const void* const* w_down,
                                  int64_t s_down, void* out, int32_t dtype, int32_t m, int64_t h, int64_t i, float eps,
                                  int32_t kind, int32_t rank, int32_t world, void* const* exchange, int32_t m_max,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  using namespace fd_host;
  if (layers < 0 || !norm_w || !w_gate_up || !w_down) return FD_ERR_ARG;
  if (world < 1 || world > kMaxTpWorld || rank < 0 || rank >= world || !exchange) return FD_ERR_ARG;
  if (m_max < 1 || m_max > MT_MAX || m > m_max) return FD_ERR_ARG;
  for (int k = 0; k < world; ++k)
    if (!exchange[k]) return FD_ERR_ARG;
  if (layers == 0) return check_mlp_args(hidden, hidden, norm_dtype, hidden, s_gu, dtype, m, h, i, kind);
  for (int l = 0; l < layers; ++l) {
    int r = check_mlp_args(hidden, norm_w[l], norm_dtype, w_gate_up[l], s_gu, dtype, m, h, i, kind);
    if (r == FD_OK) r = check_down(w_down[l], s_down, out, dtype, dtype, i);
    if (r != FD_OK) return r;
  }
  if (m == 0 || h == 0) return FD_OK;
  if (!workspace || workspace_bytes < fd_post_attn_mlp_workspace_bytes(m, h, i)) return FD_ERR_WORKSPACE;
  const Workspace ws = carve(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ping[2] = {ws.tail + align256(static_cast<size_t>(m) * i * 2),
                   ws.tail + align256(static_cast<size_t>(m) * i * 2) + align256(static_cast<size_t>(m) * h * 2)};
  const int rp = mlp_stack_persistent(hidden, layers, norm_w, norm_dtype, w_gate_up, s_gu, w_down, s_down, out,
                                      dtype, m, h, i, eps, kind, ws, ws.tail, ping[0], ping[1], st, rank, world,
                                      exchange, m_max);
  if (rp != FD_ERR_UNSUPPORTED) return rp;
  // three launches per layer (two with FD_TP_FOLD=1): fd_post_attn_mlp_tp_out
  const void* cur = hidden;
  for (int l = 0; l < layers; ++l) {
    void* dst = l == layers - 1 ? out : ping[l & 1];
    const int r = fd_post_attn_mlp_tp_out(cur, norm_w[l], norm_dtype, w_gate_up[l], s_gu, w_down[l], s_down, dst,
                                          dtype, m, h, i, eps, kind, rank, world, exchange, m_max, workspace,
                                          workspace_bytes, stream);
    if (r != FD_OK) return r;
    cur = dst;
  }
  return FD_OK;
}

int fd_post_attn_mlp_stack_out(const void* hidden, int32_t layers, const void* const* norm_w, int32_t norm_dtype,
                               const void* const* w_gate_up, int64_t s_gu, const void* const* w_down,
                               int64_t s_down, void* out, int32_t dtype, int32_t m, int64_t h, int64_t i, float eps,
                               int32_t kind, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace fd_host;
  if (layers < 0 || !norm_w || !w_gate_up || !w_down) return FD_ERR_ARG;
  if (layers == 0) return check_mlp_args(hidden, hidden, norm_dtype, hidden, s_gu, dtype, m, h, i, kind);
  for (int l = 0; l < layers; ++l) {
    int r = check_mlp_args(hidden, norm_w[l], norm_dtype, w_gate_up[l], s_gu, dtype, m, h, i, kind);
    if (r == FD_OK) r = check_down(w_down[l], s_down, out, dtype, dtype, i);
    if (r != FD_OK) return r;
  }
  if (m == 0 || h == 0) return FD_OK;
  if (!workspace || workspace_bytes < fd_post_attn_mlp_workspace_bytes(m, h, i)) return FD_ERR_WORKSPACE;
  const Workspace ws = carve(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Layer l reads h_l and writes h_{l+1}: the two ping-pong buffers behind
  // mid hold the inner activations; `out` receives only the last layer.
  char* ping[2] = {ws.tail + align256(static_cast<size_t>(m) * i * 2),
                   ws.tail + align256(static_cast<size_t>(m) * i * 2) + align256(static_cast<size_t>(m) * h * 2)};
  // One persistent kernel for the whole stack where it applies (bit-identical
  // to the chain below); otherwise two launches per layer.
  const int rp = mlp_stack_persistent(hidden, layers, norm_w, norm_dtype, w_gate_up, s_gu, w_down, s_down, out,
                                      dtype, m, h, i, eps, kind, ws, ws.tail, ping[0], ping[1], st);
  if (rp != FD_ERR_UNSUPPORTED) return rp;
  const void* cur = hidden;
  for (int l = 0; l < layers; ++l) {
    void* dst = l == layers - 1 ? out : ping[l & 1];
    const int r = mlp_layer(cur, norm_w[l], norm_dtype, w_gate_up[l], s_gu, w_down[l], s_down, dst, false, true,
                            dtype, m, h, i, eps, kind, ws, st);
    if (r != FD_OK) return r;
    cur = dst;
  }
  return FD_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- no-alloc GEMV
// fd_linear_out_noalloc runs fd_linear_out with a scratch area that lives in
// this library's own static device memory instead of a caller workspace.  It
// is for callers that have no device memory to hand over: a host that has no
// allocator of its own, or one whose memory plan is frozen after start-up and
// forbids any further device allocation.  Nothing here allocates.
//
// The scratch holds the same layout as a caller workspace (split-K slots,
// per-block counters, the status word).  Static device memory is zero when
// the library's code is loaded onto a device, which is the state the counters
// and the status word must start in; every completed launch leaves the
// counters at zero again.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t{6} << 20;  // 6 MiB per device
constexpr int kNoAllocMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Address of the current device's copy of the scratch.  Looked up once per
// device (the first call on that device) and cached.
int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return FD_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return FD_ERR_DEVICE;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return FD_OK;
}

}  // namespace

extern "C" {

size_t fd_linear_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int fd_linear_out_noalloc(const void* x, int64_t sxm, int64_t sxk, const void* w, int64_t swn, int64_t swk,
                          const void* bias, int32_t bias_dtype, int64_t sbias, const void* row_add,
                          int32_t ra_dtype, int64_t srm, int64_t srn, void* y, int64_t sym, int64_t syn,
                          int32_t dtype, int32_t m, int64_t n, int64_t k, int32_t kind, void* stream) {
  if (fd_linear_workspace_bytes(m, n, k) > kNoAllocScratchBytes) return FD_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int r = noalloc_scratch(&scratch);
  if (r != FD_OK) return r;
  return fd_linear_out(x, sxm, sxk, w, swn, swk, bias, bias_dtype, sbias, row_add, ra_dtype, srm, srn, y, sym, syn,
                       dtype, m, n, k, kind, scratch, kNoAllocScratchBytes, stream);
}

// The scratch's status word, after every call enqueued on `stream` so far:
// non-zero when a bounded in-kernel wait expired (the bits of the workspace
// status word).  Copies 4 bytes into host memory and waits for `stream`.
int fd_linear_noalloc_status(int32_t* status, void* stream) {
  if (!status) return FD_ERR_ARG;
  void* scratch = nullptr;
  const int r = noalloc_scratch(&scratch);
  if (r != FD_OK) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t v = 0;
  if (cudaMemcpyAsync(&v, static_cast<char*>(scratch) + status_offset(), sizeof(v), cudaMemcpyDeviceToHost, st) !=
          cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return FD_ERR_DEVICE;
  *status = v;
  return FD_OK;
}

// Zero the scratch's split-K counters and status word on `stream`: the state
// a launch needs.  After a call whose wait expired, counters may be left
// mid-count; this puts the scratch back in order without allocating.
int fd_linear_noalloc_reset(void* stream) {
  void* scratch = nullptr;
  const int r = noalloc_scratch(&scratch);
  if (r != FD_OK) return r;
  const size_t bytes = streamk_ws_bytes() - counters_offset();  // counters, then the status word
  return from_cuda(cudaMemsetAsync(static_cast<char*>(scratch) + counters_offset(), 0, bytes,
                                   static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
