// Small-batch GEMV family (M = 1..16) and the fused post-attention MLP.
//
// Design (sm_100a, HBM-bound: a weight byte is used 2*M times):
//  * Stream-K over the weight.  The weight is cut into blocks of 128 rows; a
//    block is a run of KS steps of B x 64 columns.  The grid (one or two CTAs
//    per SM) splits the flat step range [0, nblocks*KS) into equal contiguous
//    pieces, so every SM streams the same number of weight bytes whatever N
//    and K are.  (The reference launches cdiv(N, 64) CTAs with no split-K,
//    kernels.py:775, which leaves most of 148 SMs idle at N = 4096.)
//  * TMA pipeline.  P producer warps take turns issuing each step's B 2-D
//    tensor-map loads (cp.async.bulk.tensor, 128-byte swizzle) of a
//    [128 x 64] weight box -- and, for a plain GEMV, the [M x 64] activation
//    boxes -- into an S-stage shared-memory ring guarded by mbarriers.
//    Measured on B200: a single issuing thread keeps only about two stages in
//    flight, so several producers (or two CTAs per SM) are what let large
//    16 KB boxes saturate HBM.  Out-of-range rows and columns are zero-filled
//    by the TMA unit.
//  * Eight consumer warps own 16 weight rows each.  "dot" kind: each lane
//    reads 16 contiguous columns of its two rows (rows g and g+8, g = lane/4,
//    q = lane%4) -- conflict-free under the 128B swizzle -- and feeds four
//    mma.sync m16n8k16 per box (swap-AB: weight = A, batch = N of 8 or 16).
//    The physical columns a lane holds map to logical MMA k-indices by one
//    fixed permutation applied to both A and B, so the sum is exact.  "simt"
//    kind: the same tiles, fp32 FMAs against all M rows.
//  * Split-K partials go to per-CTA slots in a caller workspace; the last CTA
//    to finish a block (an atomic counter) sums the slots in CTA order --
//    deterministic, no inter-CTA waiting -- applies the epilogue and re-zeroes
//    the counter, so the workspace is ready for the next launch or replay.
//  * Every mbarrier wait is bounded (globaltimer, 2 s): on expiry the CTA sets
//    a bit in the workspace status word and leaves instead of hanging.
//  * The MLP gate/up kernel computes RMSNorm of the (tiny) hidden batch into
//    shared memory in its prologue; each 128-row block is 64 gate rows over
//    the matching 64 up rows (one 3-D box), so SwiGLU is a local epilogue.
//    The down kernel adds the residual in its epilogue.  Kernels launch with
//    programmatic dependent launch: the weight prefetch is issued before
//    griddepcontrol.wait.
#include "fd_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>

using namespace fd;

namespace {

constexpr int GW = 8;                      // consumer warps per CTA
constexpr int BR = GW * 16;                // weight rows per block
constexpr int KC = 64;                     // columns per box (128 bytes of a 16-bit row)
constexpr int BOX_BYTES = BR * KC * 2;     // 16 KB weight box
constexpr int MAX_BOXES = 2;               // boxes per stage
constexpr int MT_MAX = 16;                 // max batch rows
constexpr int CONSUMERS = GW * 32;
constexpr int MAX_PRODUCERS = 3;
constexpr int MAX_STAGES = 12;
constexpr int64_t kMaxCounters = 1 << 16;  // blocks per launch (N <= 8M rows)
constexpr uint64_t kWaitNs = 2000000000ull;  // bounded mbarrier waits: 2 s

// Status bits written to the workspace status word.
constexpr int kStatusFullTimeout = 1;
constexpr int kStatusEmptyTimeout = 2;

enum Mode { MODE_LINEAR = 0, MODE_GATEUP = 1 };

struct GemvArgs {
  const void* bias;
  int32_t bias_dtype;
  int64_t sbias;
  const void* ra;
  int32_t ra_dtype;
  int64_t srm, srn;
  char* y;
  int64_t sym, syn;
  int32_t y_f32;    // LINEAR mode: store fp32 instead of T (tensor-parallel partials)
  int32_t m;
  int64_t n, k;
  // stream-K geometry
  int64_t ks;       // steps per block
  int64_t nblocks;
  int64_t total;    // nblocks * ks
  int32_t stages;   // S
  int32_t boxes;    // B: 64-column boxes per step
  int32_t x_slot;   // LINEAR: bytes per activation box slot (1024-aligned)
  float* slots;     // [grid][2][BR * MT_MAX]
  int* counters;    // [nblocks]
  int* status;      // error bits
  // gate/up mode
  int64_t inner;            // I: number of gate (= up) rows
  const void* hidden;       // [m, k] rows, row stride hidden_stride
  int64_t hidden_stride;
  const void* norm_w;
  int32_t norm_dtype;
  float eps;
};

// ------------------------------------------------------------ PTX helpers
template <typename T>
FD_DEV void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                     uint32_t b1);
template <>
FD_DEV void mma16816<__nv_bfloat16>(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                    uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
FD_DEV void mma16816<__half>(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                             uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

FD_DEV uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
FD_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
FD_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
FD_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
FD_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
FD_DEV uint32_t mbar_try(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.b32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok;
}
// Wait for the phase with the given parity to complete; false after kWaitNs.
FD_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_addr(bar);
  if (mbar_try(addr, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try(addr, parity)) return true;
    if (globaltimer() - t0 > kWaitNs) return false;
  }
}
FD_DEV uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// 2-D / 3-D tiled TMA loads into this CTA's shared memory, completing on `bar`
// (no multicast: every CTA fetches its own tiles).
FD_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar,
                        uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}
FD_DEV void tma_load_3d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z, uint64_t* bar,
                        uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}
FD_DEV void tma_load_2d_plain(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}
FD_DEV void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
FD_DEV void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(CONSUMERS) : "memory"); }
FD_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
FD_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Byte offset of 16-byte chunk c of row r inside a 128B-swizzled tile whose
// rows are 128 bytes (TMA CU_TENSOR_MAP_SWIZZLE_128B, 1024-byte aligned base).
FD_DEV uint32_t swz(int r, int c) { return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4)); }

// ------------------------------------------------------------ stream-K split
FD_DEV int64_t range_start(int64_t c, int64_t total, int64_t G) { return c * total / G; }
// The CTA whose range holds step t.
FD_DEV int64_t cta_of(int64_t t, int64_t total, int64_t G) { return ((t + 1) * G - 1) / total; }

FD_DEV float silu_mul(float g, float u) {
  // Stable sigmoid, as the reference kernel computes it (kernels.py:448-451).
  const float e = expf(-fabsf(g));
  const float sig = g >= 0.f ? 1.0f / (1.0f + e) : e / (1.0f + e);
  return g * sig * u;
}

// Accumulator ownership shared by both kinds: lane (g, q) owns, for tile t and
// element e, weight row g + 8*(e>>1) of its warp and batch column
// 8t + 2q + (e&1) -- the m16n8 C-fragment layout.
template <int NT>
struct Acc {
  float v[NT][4];
  FD_DEV void zero() {
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) v[t][e] = 0.f;
  }
};

// ------------------------------------------------------------ epilogues
template <typename T, int NT, int MODE>
struct Epilogue;

// Plain linear: y = round(acc + bias + row_add)  (or the fp32 sum).
template <typename T, int NT>
struct Epilogue<T, NT, MODE_LINEAR> {
  FD_DEV static void run(const GemvArgs& a, int64_t blk, const Acc<NT>& acc, float* /*xchg*/) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t row = blk * BR + 16 * warp + g + 8 * (e >> 1);
        const int col = 8 * t + 2 * q + (e & 1);
        if (row < a.n && col < a.m) {
          float v = acc.v[t][e];
          if (a.bias) v += load_as_f32(a.bias, a.bias_dtype, row * a.sbias);
          if (a.ra) v += load_as_f32(a.ra, a.ra_dtype, col * a.srm + row * a.srn);
          if (a.y_f32)
            reinterpret_cast<float*>(a.y)[col * a.sym + row * a.syn] = v;
          else
            reinterpret_cast<T*>(a.y)[col * a.sym + row * a.syn] = from_f32<T>(v);
        }
      }
    }
  }
};

// Gate/up + SwiGLU: warps 0..3 hold gate rows, warps 4..7 the matching up rows.
// gate and up are rounded to T first, as the reference rounds gate_up
// (reference.py:390, ops.py:313), then mid = round(silu(gate) * up).
template <typename T, int NT>
struct Epilogue<T, NT, MODE_GATEUP> {
  FD_DEV static void run(const GemvArgs& a, int64_t blk, const Acc<NT>& acc, float* xchg) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    constexpr int HALF = GW / 2;
    if (warp >= HALF) {
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = 16 * (warp - HALF) + g + 8 * (e >> 1);
          const int col = 8 * t + 2 * q + (e & 1);
          xchg[r * MT_MAX + col] = acc.v[t][e];
        }
    }
    consumer_sync();
    if (warp < HALF) {
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = 16 * warp + g + 8 * (e >> 1);
          const int col = 8 * t + 2 * q + (e & 1);
          const int64_t j = blk * (BR / 2) + r;
          if (j < a.inner && col < a.m) {
            const float gt = round_to<T>(acc.v[t][e]);
            const float up = round_to<T>(xchg[r * MT_MAX + col]);
            reinterpret_cast<T*>(a.y)[col * a.sym + j] = from_f32<T>(silu_mul(gt, up));
          }
        }
    }
    consumer_sync();
  }
};

// Block `blk` ends inside this CTA's range [s0, s1): finish it directly if the
// CTA covered all of it, else publish the partial and let the last of the
// block's CTAs reduce.  Called by all consumer threads together.
template <typename T, int NT, int MODE>
FD_DEV void flush_block(const GemvArgs& a, int64_t blk, const Acc<NT>& acc, float* xchg, int64_t s0,
                        int64_t s1, int64_t G, int64_t c, int* s_last) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const bool covered = (s0 <= blk * a.ks) && (s1 >= (blk + 1) * a.ks);
  if (covered) {
    Epilogue<T, NT, MODE>::run(a, blk, acc, xchg);
    return;
  }
  const int slot = (blk == s0 / a.ks) ? 0 : 1;
  float* sp = a.slots + (c * 2 + slot) * (BR * MT_MAX);
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = 16 * warp + g + 8 * h;
      const int col = 8 * t + 2 * q;
      *reinterpret_cast<float2*>(sp + r * MT_MAX + col) = make_float2(acc.v[t][2 * h], acc.v[t][2 * h + 1]);
    }
  __threadfence();
  consumer_sync();
  const int64_t cf = cta_of(blk * a.ks, a.total, G);
  const int64_t cl = cta_of((blk + 1) * a.ks - 1, a.total, G);
  if (threadIdx.x == 0) {
    const int old = atomicAdd(a.counters + blk, 1);
    *s_last = (old == static_cast<int>(cl - cf));
  }
  consumer_sync();
  if (*s_last) {
    __threadfence();
    Acc<NT> sum;
    sum.zero();
    for (int64_t cc = cf; cc <= cl; ++cc) {
      const int sl = (blk == range_start(cc, a.total, G) / a.ks) ? 0 : 1;
      const float* rp = a.slots + (cc * 2 + sl) * (BR * MT_MAX);
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = 16 * warp + g + 8 * h;
          const int col = 8 * t + 2 * q;
          const float2 v = __ldcg(reinterpret_cast<const float2*>(rp + r * MT_MAX + col));
          sum.v[t][2 * h] += v.x;
          sum.v[t][2 * h + 1] += v.y;
        }
    }
    Epilogue<T, NT, MODE>::run(a, blk, sum, xchg);
    if (threadIdx.x == 0) a.counters[blk] = 0;
  }
}

// ------------------------------------------------------------ the TMA kernel
// KIND 0 = dot (mma.sync), 1 = simt.  MP = padded batch for simt (1..16).
// NT = number of 8-wide MMA batch tiles (1 for m <= 8, 2 for m <= 16).
// MAXT / MINB: launch bounds (threads, resident CTAs per SM).
template <typename T, int NT, int KIND, int MP, int MODE, int MAXT, int MINB>
__global__ void __launch_bounds__(MAXT, MINB)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                    const GemvArgs a) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ int s_last;
  __shared__ int s_abort;
  __shared__ float s_sumsq[GW][MT_MAX];
  // 1024-byte alignment for the 128B swizzle atoms.
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~static_cast<uintptr_t>(1023));
  const int S = a.stages;
  const int B = a.boxes;
  const int x_slot = a.x_slot;
  const int64_t w_stage = static_cast<int64_t>(B) * BOX_BYTES;
  unsigned char* wst = smem;                                  // S x B x 16 KB
  unsigned char* xst = wst + S * w_stage;                     // LINEAR: S x B x x_slot
  // GATEUP: normed x as 64-column chunks of [m rows x 128 B], swizzled like a TMA tile
  unsigned char* xs = xst;
  const int64_t x_bytes = MODE == MODE_GATEUP ? a.ks * B * a.m * 128 : static_cast<int64_t>(S) * B * x_slot;
  float* xchg = reinterpret_cast<float*>(xst + ((x_bytes + 15) & ~15ll));
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(xchg) + (BR / 2) * MT_MAX * 4);
  uint64_t* empty = full + MAX_STAGES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = static_cast<int>(blockDim.x >> 5) - GW;
  const int64_t G = gridDim.x, c = blockIdx.x;
  const int64_t s0 = range_start(c, a.total, G);
  const int64_t s1 = range_start(c + 1, a.total, G);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], GW);
    }
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp >= GW) {
    // ================= producer warps: producer p issues steps p, p+P, ...
    const int p = warp - GW;
    if (lane == 0) {
      prefetch_map(&wmap);
      if (MODE == MODE_LINEAR) prefetch_map(&xmap);
      const uint64_t pol = evict_first_policy();
      const uint32_t stage_bytes =
          static_cast<uint32_t>(w_stage) + (MODE == MODE_LINEAR ? static_cast<uint32_t>(B * a.m * 128) : 0u);
      const int64_t n_steps = s1 - s0;
      auto issue_w = [&](int64_t it) {
        const int64_t t = s0 + it;
        const int64_t b = t / a.ks, kk = t - (t / a.ks) * a.ks;
        const int s = static_cast<int>(it % S);
        unsigned char* dst = wst + s * w_stage;
        for (int j = 0; j < B; ++j) {
          const int32_t col = static_cast<int32_t>((kk * B + j) * KC);
          if (MODE == MODE_GATEUP)
            tma_load_3d(dst + j * BOX_BYTES, &wmap, col, static_cast<int32_t>(b * (BR / 2)), 0, &full[s], pol);
          else
            tma_load_2d(dst + j * BOX_BYTES, &wmap, col, static_cast<int32_t>(b * BR), &full[s], pol);
        }
      };
      auto issue_x = [&](int64_t it) {
        const int64_t t = s0 + it;
        const int64_t kk = t - (t / a.ks) * a.ks;
        const int s = static_cast<int>(it % S);
        for (int j = 0; j < B; ++j)
          tma_load_2d_plain(xst + (s * B + j) * x_slot, &xmap, static_cast<int32_t>((kk * B + j) * KC), 0, &full[s]);
      };
      const int64_t npre = n_steps < S ? n_steps : S;
      // (1) weight tiles of the first stages: independent of the previous kernel
      for (int64_t it = p; it < npre; it += P) {
        mbar_expect_tx(&full[it], stage_bytes);
        issue_w(it);
      }
      // (2) activation tiles read the previous kernel's output
      if (MODE == MODE_LINEAR) {
        grid_dep_wait();
        for (int64_t it = p; it < npre; it += P) issue_x(it);
      }
      // (3) steady state: refill a stage once all consumer warps released it
      int64_t last = -1;
      for (int64_t it = p; it < npre; it += P) last = it;
      int64_t it = p;
      while (it < npre) it += P;
      for (; it < n_steps; it += P) {
        const int s = static_cast<int>(it % S);
        if (!mbar_wait(&empty[s], static_cast<uint32_t>((it / S - 1) & 1))) {
          atomicOr(a.status, kStatusEmptyTimeout);
          break;
        }
        if (*reinterpret_cast<volatile int*>(&s_abort)) break;
        mbar_expect_tx(&full[s], stage_bytes);
        issue_w(it);
        if (MODE == MODE_LINEAR) issue_x(it);
        last = it;
      }
      // Drain: never leave the CTA with this producer's copies still landing.
      // Only the last S steps are checked: their stages are never refilled,
      // so their phase parity is unambiguous.
      for (int64_t d = last; d >= 0 && d >= n_steps - S; d -= P) {
        if (!mbar_wait(&full[d % S], static_cast<uint32_t>((d / S) & 1))) break;
      }
    }
    grid_dep_launch();
    return;
  }

  // ================= consumer warps
  const int g = lane >> 2, q = lane & 3;
  const int tid = threadIdx.x;
  grid_dep_wait();
  if (MODE == MODE_GATEUP) {
    // RMSNorm of the m hidden rows into shared memory, rounded to T
    // (reference.py:389 rounds `normed` to the activation dtype), stored as
    // 64-column chunks of [m x 128 B] with the same swizzle as a TMA tile;
    // columns past k (up to the end of the last step) are zero.
    const int nvec = static_cast<int>(a.k / 8);
    const int nvec_pad = static_cast<int>(a.ks * B * (KC / 8));
    float ss[MT_MAX];
#pragma unroll
    for (int mrow = 0; mrow < MT_MAX; ++mrow) ss[mrow] = 0.f;
    for (int v = tid; v < nvec; v += CONSUMERS) {
#pragma unroll
      for (int mrow = 0; mrow < MT_MAX; ++mrow) {
        if (mrow < a.m) {
          const uint4* hr =
              reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.hidden) + mrow * a.hidden_stride);
          float f[8];
          unpack8<T>(__ldg(hr + v), f);
#pragma unroll
          for (int e = 0; e < 8; ++e) ss[mrow] += f[e] * f[e];
        }
      }
    }
#pragma unroll
    for (int mrow = 0; mrow < MT_MAX; ++mrow) {
      if (mrow < a.m) {
        const float t = warp_sum(ss[mrow]);
        if (lane == 0) s_sumsq[warp][mrow] = t;
      }
    }
    consumer_sync();
    float inv[MT_MAX];
#pragma unroll
    for (int mrow = 0; mrow < MT_MAX; ++mrow) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < GW; ++w) tot += mrow < a.m ? s_sumsq[w][mrow] : 0.f;
      inv[mrow] = 1.0f / sqrtf(tot / static_cast<float>(a.k) + a.eps);
    }
    const int wes = a.norm_dtype == FD_F32 ? 4 : 2;
    for (int v = tid; v < nvec_pad; v += CONSUMERS) {
      const int chunk = v >> 3, cc = v & 7;
      float wv[8];
      if (v < nvec) load8_as_f32(static_cast<const char*>(a.norm_w) + static_cast<int64_t>(v) * 8 * wes, a.norm_dtype, wv);
#pragma unroll
      for (int mrow = 0; mrow < MT_MAX; ++mrow) {
        if (mrow < a.m) {
          uint4 packed = make_uint4(0, 0, 0, 0);
          if (v < nvec) {
            const uint4* hr =
                reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.hidden) + mrow * a.hidden_stride);
            float f[8], o[8];
            unpack8<T>(__ldg(hr + v), f);
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = f[e] * inv[mrow] * wv[e];
            packed = pack8<T>(o);
          }
          *reinterpret_cast<uint4*>(xs + (static_cast<int64_t>(chunk) * a.m + mrow) * 128 +
                                    ((cc ^ (mrow & 7)) << 4)) = packed;
        }
      }
    }
    consumer_sync();
  }
  grid_dep_launch();

  Acc<NT> acc;
  acc.zero();
  float sacc[2][MP];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int mm = 0; mm < MP; ++mm) sacc[r][mm] = 0.f;

  const int r0 = 16 * warp + g;  // weight rows of this lane in every box: r0, r0 + 8
  int64_t cb = s0 / a.ks, ck = s0 - (s0 / a.ks) * a.ks;
  for (int64_t it = 0; it < s1 - s0; ++it) {
    const int s = static_cast<int>(it % S);
    if (!mbar_wait(&full[s], static_cast<uint32_t>((it / S) & 1))) {
      atomicOr(a.status, kStatusFullTimeout);
      s_abort = 1;
      return;  // every consumer warp times out on this same stage
    }
    uint4 wa[MAX_BOXES][2], wb[MAX_BOXES][2];
#pragma unroll
    for (int j = 0; j < MAX_BOXES; ++j) {
      if (j < B) {
        const unsigned char* wt = wst + s * w_stage + j * BOX_BYTES;
        wa[j][0] = *reinterpret_cast<const uint4*>(wt + swz(r0, 2 * q));
        wa[j][1] = *reinterpret_cast<const uint4*>(wt + swz(r0, 2 * q + 1));
        wb[j][0] = *reinterpret_cast<const uint4*>(wt + swz(r0 + 8, 2 * q));
        wb[j][1] = *reinterpret_cast<const uint4*>(wt + swz(r0 + 8, 2 * q + 1));
      }
    }
    // activation box j of this step: [m rows x 128 B] (swizzled by row & 7)
    auto xbox = [&](int j) -> const unsigned char* {
      return MODE == MODE_LINEAR ? xst + (s * B + j) * x_slot : xs + ((ck * B + j) * a.m) * 128;
    };
    if (KIND == 0) {
      uint4 xa[MAX_BOXES][NT][2];
#pragma unroll
      for (int j = 0; j < MAX_BOXES; ++j) {
        if (j < B) {
          const unsigned char* xt = xbox(j);
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const int n = g + 8 * t;
            if (n < a.m) {
              xa[j][t][0] = *reinterpret_cast<const uint4*>(xt + swz(n, 2 * q));
              xa[j][t][1] = *reinterpret_cast<const uint4*>(xt + swz(n, 2 * q + 1));
            } else {
              xa[j][t][0] = make_uint4(0, 0, 0, 0);
              xa[j][t][1] = make_uint4(0, 0, 0, 0);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      // physical column 16q + 4h + j  <->  logical k of MMA h: (2q, 2q+1, 2q+8, 2q+9)
#pragma unroll
      for (int j = 0; j < MAX_BOXES; ++j) {
        if (j < B) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            mma16816<T>(acc.v[t], wa[j][0].x, wb[j][0].x, wa[j][0].y, wb[j][0].y, xa[j][t][0].x, xa[j][t][0].y);
            mma16816<T>(acc.v[t], wa[j][0].z, wb[j][0].z, wa[j][0].w, wb[j][0].w, xa[j][t][0].z, xa[j][t][0].w);
            mma16816<T>(acc.v[t], wa[j][1].x, wb[j][1].x, wa[j][1].y, wb[j][1].y, xa[j][t][1].x, xa[j][t][1].y);
            mma16816<T>(acc.v[t], wa[j][1].z, wb[j][1].z, wa[j][1].w, wb[j][1].w, xa[j][t][1].z, xa[j][t][1].w);
          }
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < MAX_BOXES; ++j) {
        if (j < B) {
          float wf[2][16];
          unpack8<T>(wa[j][0], wf[0]);
          unpack8<T>(wa[j][1], wf[0] + 8);
          unpack8<T>(wb[j][0], wf[1]);
          unpack8<T>(wb[j][1], wf[1] + 8);
          const unsigned char* xt = xbox(j);
#pragma unroll
          for (int mm = 0; mm < MP; ++mm) {
            if (mm < a.m) {
              float xf[16];
              unpack8<T>(*reinterpret_cast<const uint4*>(xt + swz(mm, 2 * q)), xf);
              unpack8<T>(*reinterpret_cast<const uint4*>(xt + swz(mm, 2 * q + 1)), xf + 8);
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                sacc[0][mm] = fmaf(wf[0][e], xf[e], sacc[0][mm]);
                sacc[1][mm] = fmaf(wf[1][e], xf[e], sacc[1][mm]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // ---- block finished (or range ends): flush
    ++ck;
    if (ck == a.ks || it + 1 == s1 - s0) {
      if (KIND == 1) {
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
          for (int mm = 0; mm < MP; ++mm) {
            float v = sacc[r][mm];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            sacc[r][mm] = v;
          }
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float v = 0.f;
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
              const int col = 8 * t + 2 * qq + (e & 1);
              if (col < MP && qq == q) v = sacc[e >> 1][col];
            }
            acc.v[t][e] = v;
          }
      }
      flush_block<T, NT, MODE>(a, cb, acc, xchg, s0, s1, G, c, &s_last);
      acc.zero();
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int mm = 0; mm < MP; ++mm) sacc[r][mm] = 0.f;
      ck = 0;
      ++cb;
    }
  }
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
size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

constexpr int kMaxCtasPerSm = 2;
int64_t max_grid() { return static_cast<int64_t>(fd_host::sm_count()) * kMaxCtasPerSm; }

// Workspace layout (fixed for a device, whatever the shape, so one buffer can
// serve every launch):  [slots: max grid x 2 x BR x MT_MAX floats]
//                       [counters: kMaxCounters ints][status: 64 ints]
//                       [MLP intermediate]
size_t slots_bytes() { return align256(static_cast<size_t>(max_grid()) * 2 * BR * MT_MAX * sizeof(float)); }
size_t counters_offset() { return slots_bytes(); }
size_t status_offset() { return counters_offset() + kMaxCounters * sizeof(int); }
size_t streamk_ws_bytes() { return status_offset() + 256; }

struct Workspace {
  float* slots;
  int* counters;
  int* status;
  char* tail;
};
Workspace carve(void* ws) {
  char* p = static_cast<char*>(ws);
  return {reinterpret_cast<float*>(p), reinterpret_cast<int*>(p + counters_offset()),
          reinterpret_cast<int*>(p + status_offset()), p + streamk_ws_bytes()};
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Tensor map over 16-bit data: `rank` dims (innermost first) with byte strides
// of the outer dims; boxes of 64 innermost elements, 128B swizzle, elements
// outside the tensor read as 0.
bool make_map(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
              const cuuint32_t* box) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, rank, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// [rows, cols] matrix with row stride `stride` elements, boxes of [box_rows x 64].
bool make_map_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t stride, int box_rows) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(KC), static_cast<cuuint32_t>(box_rows)};
  return make_map(map, base, 2, dims, strides, box);
}

int x_slot_bytes(int m) { return m <= 8 ? 1024 : 2048; }

size_t tma_smem_bytes(int mode, int m, int64_t ks, int stages, int boxes) {
  const size_t xbytes = mode == MODE_GATEUP ? static_cast<size_t>(ks) * boxes * m * 128
                                            : static_cast<size_t>(stages) * boxes * x_slot_bytes(m);
  return 1024 + static_cast<size_t>(stages) * boxes * BOX_BYTES + ((xbytes + 15) & ~static_cast<size_t>(15)) +
         (BR / 2) * MT_MAX * 4 + 2 * MAX_STAGES * 8;
}

constexpr size_t kSmemPerSm = 228 * 1024;          // shared memory of one SM
constexpr size_t kSmemPerCta = 227 * 1024 - 1024;  // opt-in maximum, less static shared memory

// Pipeline geometry of one launch: CTAs per SM, producer warps, 64-column
// boxes per step and ring stages.  Measured on B200 over the Llama-3-8B MLP
// shapes (32-launch CUDA graphs, M = 1 and 8): one CTA per SM with two
// producer warps, 32 KB steps (two boxes) and four stages streamed fastest
// (gate/up 5.0 TB/s, down 4.5 TB/s); two CTAs per SM with one producer each
// were 3-10% slower, 16 KB steps 20-30% slower.
struct Geometry {
  int ctas_per_sm, producers, boxes, stages;
};

Geometry choose_geometry(int mode, int m, int64_t k) {
  Geometry g{1, 2, 2, 4};
  if (const char* env = std::getenv("FD_GEMV_GEOMETRY")) {  // tuning override: "cps,producers,boxes,stages"
    int a = 0, b = 0, c = 0, d = 0;
    if (std::sscanf(env, "%d,%d,%d,%d", &a, &b, &c, &d) == 4 && a >= 1 && a <= 2 && b >= 1 &&
        b <= MAX_PRODUCERS && c >= 1 && c <= MAX_BOXES && d >= 2 && d <= MAX_STAGES)
      g = {a, b, c, d};
  }
  const int64_t step_cols = static_cast<int64_t>(g.boxes) * KC;
  const int64_t ks = (k + step_cols - 1) / step_cols;
  const size_t per_cta = g.ctas_per_sm == 2 ? kSmemPerSm / 2 - 2048 : kSmemPerCta;
  while (g.stages > 2 && tma_smem_bytes(mode, m, ks, g.stages, g.boxes) > per_cta) --g.stages;
  if (tma_smem_bytes(mode, m, ks, g.stages, g.boxes) > per_cta && g.ctas_per_sm == 2) {
    // Two CTAs do not fit (a wide normalised batch): one CTA, two producers.
    g.ctas_per_sm = 1;
    g.producers = std::max(g.producers, 2);
    g.stages = MAX_STAGES;
    while (g.stages > 2 && tma_smem_bytes(mode, m, ks, g.stages, g.boxes) > kSmemPerCta) --g.stages;
  }
  if (g.ctas_per_sm == 2) g.producers = 1;  // the two-CTA kernels are built for 288 threads
  g.stages -= g.stages % g.producers;       // every stage is always refilled by the same producer
  if (g.stages < 2 || tma_smem_bytes(mode, m, ks, g.stages, g.boxes) > kSmemPerCta) g.stages = 0;
  return g;
}

template <typename Kern>
cudaError_t launch_tma(Kern kern, const CUtensorMap& wm, const CUtensorMap& xm, const GemvArgs& a,
                       const Geometry& geo, size_t smem, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int64_t grid =
      std::max<int64_t>(1, std::min<int64_t>(static_cast<int64_t>(fd_host::sm_count()) * geo.ctas_per_sm, a.total));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(CONSUMERS + 32 * geo.producers);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, wm, xm, a);
}

template <typename T, int MODE, int NT, int KIND, int MP>
cudaError_t launch_geo(const CUtensorMap& wm, const CUtensorMap& xm, const GemvArgs& a, const Geometry& geo,
                       size_t smem, cudaStream_t st) {
  if (geo.ctas_per_sm == 2)
    return launch_tma(gemv_tma_kernel<T, NT, KIND, MP, MODE, CONSUMERS + 32, 2>, wm, xm, a, geo, smem, st);
  return launch_tma(gemv_tma_kernel<T, NT, KIND, MP, MODE, CONSUMERS + 32 * MAX_PRODUCERS, 1>, wm, xm, a, geo,
                    smem, st);
}

template <typename T, int MODE>
cudaError_t dispatch_tma(const CUtensorMap& wm, const CUtensorMap& xm, const GemvArgs& a, int kind,
                         const Geometry& geo, size_t smem, cudaStream_t st) {
  if (kind == FD_KIND_DOT) {
    if (a.m <= 8) return launch_geo<T, MODE, 1, 0, 1>(wm, xm, a, geo, smem, st);
    return launch_geo<T, MODE, 2, 0, 1>(wm, xm, a, geo, smem, st);
  }
  // simt: one CTA per SM (its accumulators need the registers)
  Geometry g1 = geo;
  if (g1.ctas_per_sm == 2) {
    g1.ctas_per_sm = 1;
    g1.producers = 2;
  }
  auto L = [&](auto kern) { return launch_tma(kern, wm, xm, a, g1, smem, st); };
  constexpr int MT1 = CONSUMERS + 32 * MAX_PRODUCERS;
  if (a.m <= 1) return L(gemv_tma_kernel<T, 1, 1, 1, MODE, MT1, 1>);
  if (a.m <= 2) return L(gemv_tma_kernel<T, 1, 1, 2, MODE, MT1, 1>);
  if (a.m <= 4) return L(gemv_tma_kernel<T, 1, 1, 4, MODE, MT1, 1>);
  if (a.m <= 8) return L(gemv_tma_kernel<T, 1, 1, 8, MODE, MT1, 1>);
  return L(gemv_tma_kernel<T, 2, 1, 16, MODE, MT1, 1>);
}

int from_cuda(cudaError_t e) { return e == cudaSuccess ? FD_OK : FD_ERR_LAUNCH; }

// Launch the stream-K TMA GEMV in LINEAR mode: y = x @ w^T (+bias)(+row_add).
int launch_linear(const void* x, int64_t sxm, const void* w, int64_t swn, GemvArgs a, int dtype, int kind,
                  const Workspace& ws, cudaStream_t st) {
  const Geometry geo = choose_geometry(MODE_LINEAR, a.m, a.k);
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
  const size_t smem = tma_smem_bytes(MODE_LINEAR, a.m, a.ks, a.stages, a.boxes);
  cudaError_t e = dtype == FD_BF16 ? dispatch_tma<__nv_bfloat16, MODE_LINEAR>(wm, xm, a, kind, geo, smem, st)
                                   : dispatch_tma<__half, MODE_LINEAR>(wm, xm, a, kind, geo, smem, st);
  return from_cuda(e);
}

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
  if (m > 0 && choose_geometry(MODE_GATEUP, m, h).stages == 0) return FD_ERR_UNSUPPORTED;
  if ((i + BR / 2 - 1) / (BR / 2) > kMaxCounters) return FD_ERR_UNSUPPORTED;
  return FD_OK;
}

// Kernel 1 of the MLP: RMSNorm (prologue) -> gate/up GEMV -> SwiGLU -> mid.
int launch_gate_up(const void* hidden, const void* norm_w, int32_t norm_dtype, const void* w_gate_up,
                   int64_t s_gu, void* mid, int64_t s_mid, int32_t dtype, int32_t m, int64_t h, int64_t i,
                   float eps, int32_t kind, const Workspace& ws, cudaStream_t st) {
  const Geometry geo = choose_geometry(MODE_GATEUP, m, h);
  if (geo.stages == 0) return FD_ERR_UNSUPPORTED;
  GemvArgs a = {};
  a.y = static_cast<char*>(mid); a.sym = s_mid; a.syn = 1;
  a.m = m; a.n = 2 * i; a.k = h;
  a.boxes = geo.boxes;
  a.stages = geo.stages;
  a.ks = (h + static_cast<int64_t>(geo.boxes) * KC - 1) / (static_cast<int64_t>(geo.boxes) * KC);
  a.nblocks = (i + BR / 2 - 1) / (BR / 2);
  a.total = a.nblocks * a.ks;
  a.slots = ws.slots; a.counters = ws.counters; a.status = ws.status;
  a.inner = i;
  a.hidden = hidden; a.hidden_stride = h;
  a.norm_w = norm_w; a.norm_dtype = norm_dtype; a.eps = eps;
  // 3-D view [2][i][h] of w_gate_up: plane 0 = gate rows, plane 1 = up rows;
  // one [2 x 64 x 64] box is 64 gate rows over the matching 64 up rows.
  CUtensorMap gm;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(h), static_cast<cuuint64_t>(i), 2};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(s_gu) * 2, static_cast<cuuint64_t>(i) * s_gu * 2};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(KC), BR / 2, 2};
  if (!make_map(&gm, w_gate_up, 3, dims, strides, box)) return FD_ERR_LAUNCH;
  const size_t smem = tma_smem_bytes(MODE_GATEUP, m, a.ks, a.stages, a.boxes);
  cudaError_t e = dtype == FD_BF16 ? dispatch_tma<__nv_bfloat16, MODE_GATEUP>(gm, gm, a, kind, geo, smem, st)
                                   : dispatch_tma<__half, MODE_GATEUP>(gm, gm, a, kind, geo, smem, st);
  return from_cuda(e);
}

}  // namespace

extern "C" {

size_t fd_linear_workspace_bytes(int32_t m, int64_t n, int64_t k) {
  (void)m;
  (void)n;
  (void)k;
  return streamk_ws_bytes();
}

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

size_t fd_post_attn_mlp_workspace_bytes(int32_t m, int64_t h, int64_t i) {
  (void)h;
  return streamk_ws_bytes() + align256(static_cast<size_t>(std::max(m, 1)) * i * 2);
}

size_t fd_workspace_status_offset(void) { return status_offset(); }

int fd_mlp_gate_up_out(const void* hidden, const void* norm_w, int32_t norm_dtype, const void* w_gate_up,
                       int64_t s_gu, void* mid, int32_t dtype, int32_t m, int64_t h, int64_t i, float eps,
                       int32_t kind, void* workspace, size_t workspace_bytes, void* stream) {
  const int chk = check_mlp_args(hidden, norm_w, norm_dtype, w_gate_up, s_gu, dtype, m, h, i, kind);
  if (chk != FD_OK) return chk;
  if (m == 0 || h == 0) return FD_OK;
  if (!mid) return FD_ERR_ARG;
  if (!workspace || workspace_bytes < streamk_ws_bytes()) return FD_ERR_WORKSPACE;
  if (!encode_fn()) return FD_ERR_DEVICE;
  return launch_gate_up(hidden, norm_w, norm_dtype, w_gate_up, s_gu, mid, i, dtype, m, h, i, eps, kind,
                        carve(workspace), static_cast<cudaStream_t>(stream));
}

int fd_post_attn_mlp_out(const void* hidden, const void* norm_w, int32_t norm_dtype, const void* w_gate_up,
                         int64_t s_gu, const void* w_down, int64_t s_down, void* out, int32_t out_dtype,
                         int32_t dtype, int32_t m, int64_t h, int64_t i, float eps, int32_t kind,
                         int32_t add_residual, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace fd_host;
  const int chk = check_mlp_args(hidden, norm_w, norm_dtype, w_gate_up, s_gu, dtype, m, h, i, kind);
  if (chk != FD_OK) return chk;
  if (m == 0 || h == 0) return FD_OK;
  if (!w_down || !out) return FD_ERR_ARG;
  if (!(out_dtype == dtype || out_dtype == FD_F32)) return FD_ERR_ARG;
  if (s_down % 8 || s_down < i || !aligned16(w_down)) return FD_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < fd_post_attn_mlp_workspace_bytes(m, h, i)) return FD_ERR_WORKSPACE;
  if (!encode_fn()) return FD_ERR_DEVICE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const Workspace ws = carve(workspace);
  char* mid = ws.tail;

  int r = launch_gate_up(hidden, norm_w, norm_dtype, w_gate_up, s_gu, mid, i, dtype, m, h, i, eps, kind, ws, st);
  if (r != FD_OK) return r;

  // Kernel 2: down GEMV (+ residual) -> out [m, h].
  GemvArgs b = {};
  b.ra = add_residual ? hidden : nullptr; b.ra_dtype = dtype; b.srm = h; b.srn = 1;
  b.y = static_cast<char*>(out); b.sym = h; b.syn = 1;
  b.y_f32 = out_dtype == FD_F32;
  b.m = m; b.n = h; b.k = i;
  return launch_linear(mid, i, w_down, s_down, b, dtype, kind, ws, st);
}

}  // extern "C"
