// The weight-streaming engine of the decode GEMV kernels (fd_gemv.cu): a plain
// linear and the MLP's gate/up stage run the same producer/consumer phases.
//
//  * Stream-K over a weight.  The weight is cut into blocks of 128 rows; a
//    block is a run of KS steps of B x 64 columns.  Every CTA of the grid owns
//    an equal contiguous piece of the flat step range [0, nblocks*KS), so
//    every SM streams the same number of weight bytes whatever N and K are.
//  * TMA ring.  P producer warps take turns issuing each step's B 2-D/3-D
//    tensor-map loads (cp.async.bulk.tensor, 128-byte swizzle, per-CTA tiles)
//    of a [128 x 64] weight box -- and, for a plain GEMV, the [M x 64]
//    activation boxes -- into an S-stage shared-memory ring guarded by
//    mbarriers (full: data landed, empty: all consumer warps read it).
//    Measured on B200: one issuing thread keeps only about two stages in
//    flight, so two producer warps with 32 KB steps are what saturate HBM.
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
//    A block that ends in the middle of a CTA's range is published by a
//    separate announcer warp, so the consumer warps never stop streaming for
//    the fence and counter round trips (measured: CTAs crossing a block
//    boundary otherwise finished 3-4 us after the others).
//  * Every wait is bounded (globaltimer): on expiry the CTA sets a bit in the
//    workspace status word and leaves instead of hanging.
#pragma once

#include "fd_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>

namespace fd_stream {

using namespace fd;

constexpr int GW = 8;                      // consumer warps per CTA
constexpr int BR = GW * 16;                // weight rows per block
constexpr int KC = 64;                     // columns per box (128 bytes of a 16-bit row)
constexpr int BOX_BYTES = BR * KC * 2;     // 16 KB weight box
constexpr int MAX_BOXES = 2;               // boxes per step
constexpr int MT_MAX = 16;                 // max batch rows
constexpr int CONSUMERS = GW * 32;
constexpr int MAX_PRODUCERS = 3;
constexpr int MAX_STAGES = 12;
constexpr int64_t kMaxCounters = 1 << 16;  // blocks per launch (N <= 8M rows)
constexpr uint64_t kWaitNs = 2000000000ull;      // bounded mbarrier waits: 2 s

// Status bits written to the workspace status word.
constexpr int kStatusFullTimeout = 1;
constexpr int kStatusEmptyTimeout = 2;

// LINEAR: a GEMV whose activation boxes arrive by TMA with the weight boxes.
// GATEUP: the MLP gate/up stage; the normalised batch is held in shared memory.
// LINEAR_X: a GEMV whose activation columns for the CTA's step range were
// staged in shared memory by the consumers (the persistent MLP stack's down
// projection: its activation is written inside the same kernel).
// MODE_LINEAR_TP: LINEAR whose epilogue also sums the tensor-parallel ranks
// (tp_fold_block) -- its own instantiations, so the plain LINEAR kernels
// carry none of that code.  MODE_GATEUP_S: GATEUP whose normalised batch was
// written by norm_rows_kernel and streams in [m x 64] boxes by TMA with each
// weight step, instead of being normalised into shared memory whole (which
// leaves too few ring stages for wide or tall batches).
enum Mode { MODE_LINEAR = 0, MODE_GATEUP = 1, MODE_LINEAR_X = 2, MODE_LINEAR_TP = 3, MODE_GATEUP_S = 4 };
__host__ __device__ constexpr bool linear_mode(int mode) { return mode == MODE_LINEAR || mode == MODE_LINEAR_TP; }
__host__ __device__ constexpr bool gateup_mode(int mode) { return mode == MODE_GATEUP || mode == MODE_GATEUP_S; }
// activation boxes stream through per-stage slots with the weight boxes
__host__ __device__ constexpr bool streams_x(int mode) { return linear_mode(mode) || mode == MODE_GATEUP_S; }

// One phase of streaming: a GEMV (LINEAR) or the MLP gate/up stage (GATEUP).
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
  // tensor-parallel exchange (LINEAR mode, tp_world > 0): each finished
  // block's fp32 partial goes to every rank's exchange buffer, followed by a
  // flag, instead of to y (layout: TpLayout in fd_common.cuh)
  char* tp_peer[kMaxTpWorld];
  int32_t tp_rank, tp_world, tp_mmax;
  int64_t tp_data_off;
  const int* tp_seq;  // this rank's round number
  // cluster split (gemv_cluster_kernel): each block's K steps are divided
  // among cl_split CTAs of one thread-block cluster, whose rings are filled
  // by cl_producers producer warps
  int32_t cl_split, cl_producers;
  // GATEUP stream-K: shared memory after the ring holds the final block's
  // later contributors' partials, staged by the announcer warp (fin_stage_ok)
  int32_t fin_stage;
};

// ------------------------------------------------------------ PTX helpers
template <typename T>
FD_DEV void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1);
template <>
FD_DEV void mma16816<__nv_bfloat16>(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                    uint32_t b1) {
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

FD_DEV uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
FD_DEV void st_shared16(void* p, const uint4& v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_addr(p)), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
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
// As mbar_try, with acquire at cluster scope: for data other CTAs of the
// cluster wrote with st.async against this mbarrier.
FD_DEV uint32_t mbar_try_cluster(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n selp.b32 %0, 1, 0, p;\n}"
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
// mbar_wait for a barrier completed by other CTAs' st.async (acquire.cluster).
FD_DEV bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_addr(bar);
  if (mbar_try_cluster(addr, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_cluster(addr, parity)) return true;
    if (globaltimer() - t0 > kWaitNs) return false;
  }
}
FD_DEV uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// 2-D / 3-D tiled TMA loads into this CTA's shared memory, completing on `bar`
// (every CTA fetches its own tiles into its own shared memory).
FD_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar, uint64_t policy) {
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
// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`
// (both addresses 16-byte aligned, bytes a multiple of 16).
FD_DEV void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
FD_DEV int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
FD_DEV void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
FD_DEV void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(CONSUMERS) : "memory"); }

// ---- thread-block clusters (the CTAs of one cluster share distributed shared memory)
FD_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of this CTA's shared-memory location `p` in cluster CTA `rank`.
FD_DEV uint32_t cluster_map(const void* p, uint32_t rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_addr(p)), "r"(rank));
  return ra;
}
FD_DEV void st_cluster_f2(uint32_t addr, float a, float b) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
// Asynchronous store of two floats to the shared::cluster address `addr`,
// counted (8 bytes) on the mbarrier at shared::cluster address `bar` in the
// same CTA: the receiver learns of the data from the mbarrier alone.
FD_DEV void st_async_f2(uint32_t addr, float a, float b, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(addr),
               "f"(a), "f"(b), "r"(bar)
               : "memory");
}
// Every thread of every CTA of the cluster takes part in each arrive / wait
// pair (the hardware barrier counts threads, so no thread may skip one).
FD_DEV void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
FD_DEV void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
FD_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Byte offset of 16-byte chunk c of row r inside a 128B-swizzled tile whose
// rows are 128 bytes (TMA CU_TENSOR_MAP_SWIZZLE_128B, 1024-byte aligned base).
FD_DEV uint32_t swz(int r, int c) { return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4)); }

// ------------------------------------------------------------ stream-K split
FD_DEV int64_t range_start(int64_t c, int64_t total, int64_t G) { return c * total / G; }
// The CTA whose range holds step t.
FD_DEV int64_t cta_of(int64_t t, int64_t total, int64_t G) { return ((t + 1) * G - 1) / total; }

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
FD_DEV void st_tagged_sys(void* p, float v, int tag) {
  asm volatile("st.relaxed.sys.global.v2.b32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(tag)
               : "memory");
}

// Tensor-parallel publication of block blk's fp32 partial (rows of this
// rank's down-projection shard, no residual): every element goes to every
// rank's exchange buffer -- peers' through NVLink peer mappings -- as a word
// tagged with the round number (layout: TpLayout).  No fence, no flag.
template <int NT>
FD_DEV void tp_publish(const GemvArgs& a, int64_t blk, const Acc<NT>& acc, int seq) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t slab = static_cast<int64_t>((seq & 1) * a.tp_world + a.tp_rank) * a.tp_mmax * a.n;
  for (int rk = 0; rk < a.tp_world; ++rk) {
    uint2* d = reinterpret_cast<uint2*>(a.tp_peer[rk] + a.tp_data_off) + slab;
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t row = blk * BR + 16 * warp + g + 8 * (e >> 1);
        const int col = 8 * t + 2 * q + (e & 1);
        if (row < a.n && col < a.m) st_tagged_sys(d + col * a.n + row, acc.v[t][e], seq + 1);
      }
  }
}

// Tensor parallel with the rank sum folded into the down projection: after
// publishing block blk, the CTA that finished it waits (bounded) for every
// other rank's tagged words of the same elements in this rank's buffer, sums
// the ranks in rank order -- its own partial from registers, the very value
// it published -- adds the residual `ex` and rounds into y: the bits
// tp_reduce_kernel would produce, without its launch.  The last block
// finished on this rank advances the round number.  All consumer threads.
// A thread's elements go in two batches of one column parity each (rows g
// and g + 8), every rank's word of a batch requested before any is checked:
// one round trip per batch, and none for a batch past the last column (at
// M = 1 the odd columns), with half the loads in flight a whole tile would
// hold in registers.
template <typename T, int NT>
FD_DEV void tp_fold_block(const GemvArgs& a, int64_t blk, const Acc<NT>& acc, const Acc<NT>& ex, int seq) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int world = a.tp_world, me = a.tp_rank;
  const int64_t rank_stride = static_cast<int64_t>(a.tp_mmax) * a.n;
  const uint2* base = reinterpret_cast<const uint2*>(a.tp_peer[me] + a.tp_data_off) +
                      static_cast<int64_t>((seq & 1) * world) * rank_stride;
  const uint32_t tag = static_cast<uint32_t>(seq + 1);
  bool ok = true;
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int par = 0; par < 2; ++par) {
      const int col = 8 * t + 2 * q + par;
      if (col >= a.m) continue;
      int64_t off[2];
      bool valid[2];
      uint2 v[2][kMaxTpWorld];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t row = blk * BR + 16 * warp + g + 8 * h;
        valid[h] = row < a.n;
        off[h] = col * a.n + row;
#pragma unroll
        for (int rk = 0; rk < kMaxTpWorld; ++rk)
          v[h][rk] = (valid[h] && rk < world && rk != me) ? ld_tagged_sys(base + rk * rank_stride + off[h])
                                                          : make_uint2(0u, tag);
      }
      const uint64_t t0 = globaltimer();
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int rk = 0; rk < kMaxTpWorld; ++rk)
          while (ok && v[h][rk].y != tag) {
            if (globaltimer() - t0 > kWaitNs) {
              atomicOr(a.status, kStatusTpTimeout);
              ok = false;
              break;
            }
            __nanosleep(32);
            v[h][rk] = ld_tagged_sys(base + rk * rank_stride + off[h]);
          }
      if (!ok) continue;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (!valid[h]) continue;
        const int e = 2 * h + par;
        float sum = 0.f;
#pragma unroll
        for (int rk = 0; rk < kMaxTpWorld; ++rk)  // rank order: the same sum on every rank
          if (rk < world) sum += rk == me ? acc.v[t][e] : __uint_as_float(v[h][rk].x);
        sum += ex.v[t][e];
        const int64_t row = blk * BR + 16 * warp + g + 8 * h;
        reinterpret_cast<T*>(a.y)[col * a.sym + row * a.syn] = from_f32<T>(sum);
      }
    }
  // every consumer thread has read the round number: count the block
  consumer_sync();
  if (threadIdx.x == 0) {
    int* seqp = reinterpret_cast<int*>(a.tp_peer[me]);
    __threadfence();
    if (atomicAdd(seqp + 1, 1) == static_cast<int>(a.nblocks) - 1) {
      seqp[1] = 0;
      *reinterpret_cast<volatile int*>(seqp) = seq + 1;
    }
  }
}

template <typename T, int NT, int MODE>
struct Epilogue;

// Plain linear: y = round(acc + bias + row_add)  (or the fp32 sum).  The
// addends are loaded by extras() -- ahead of time where the caller can, so
// their memory round trip overlaps the split-K bookkeeping.
template <typename T, int NT>
struct Epilogue<T, NT, MODE_LINEAR> {
  FD_DEV static void extras(const GemvArgs& a, int64_t blk, Acc<NT>& ex) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t row = blk * BR + 16 * warp + g + 8 * (e >> 1);
        const int col = 8 * t + 2 * q + (e & 1);
        float v = 0.f;
        if (row < a.n && col < a.m) {
          if (a.bias) v += load_as_f32(a.bias, a.bias_dtype, row * a.sbias);
          // row_add may have been written by an earlier kernel: read through L2
          if (a.ra) v += load_as_f32_cg(a.ra, a.ra_dtype, col * a.srm + row * a.srn);
        }
        ex.v[t][e] = v;
      }
    }
  }
  FD_DEV static void run(const GemvArgs& a, int64_t blk, const Acc<NT>& acc, const Acc<NT>& ex, float* /*xchg*/) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    if (a.tp_world > 0) {
      tp_publish(a, blk, acc, *reinterpret_cast<const volatile int*>(a.tp_seq));
      return;
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t row = blk * BR + 16 * warp + g + 8 * (e >> 1);
        const int col = 8 * t + 2 * q + (e & 1);
        if (row < a.n && col < a.m) {
          const float v = acc.v[t][e] + ex.v[t][e];
          if (a.y_f32)
            reinterpret_cast<float*>(a.y)[col * a.sym + row * a.syn] = v;
          else
            reinterpret_cast<T*>(a.y)[col * a.sym + row * a.syn] = from_f32<T>(v);
        }
      }
    }
  }
};

// Tensor parallel with the rank sum folded in: publish the block's partial
// to every rank, then sum the ranks' words + the residual (`ex`, from ra)
// into y (tp_fold_block).
template <typename T, int NT>
struct Epilogue<T, NT, MODE_LINEAR_TP> {
  FD_DEV static void extras(const GemvArgs& a, int64_t blk, Acc<NT>& ex) {
    Epilogue<T, NT, MODE_LINEAR>::extras(a, blk, ex);
  }
  FD_DEV static void run(const GemvArgs& a, int64_t blk, const Acc<NT>& acc, const Acc<NT>& ex, float* /*xchg*/) {
    const int seq = *reinterpret_cast<const volatile int*>(a.tp_seq);
    tp_publish(a, blk, acc, seq);
    tp_fold_block<T, NT>(a, blk, acc, ex, seq);
  }
};

// The persistent MLP stack's per-layer pointers: its consumers set them at
// the start of each phase (one shared copy per CTA), so the phase's GemvArgs
// stay in kernel parameter space -- read as constant operands, holding no
// registers in the streaming loop -- while the layer changes.
__shared__ const void* sx_ra;  // LINEAR_X: the residual rows added in the epilogue
__shared__ char* sx_y;         // LINEAR_X: the output rows
__shared__ int sx_seq;         // LINEAR_X, tensor parallel: the layer's exchange round

// LINEAR_X: y = round(acc + row_add), with row_add and y from sx_ra / sx_y
// (the stack's down projection: no bias, 16-bit output).
template <typename T, int NT>
struct Epilogue<T, NT, MODE_LINEAR_X> {
  FD_DEV static void extras(const GemvArgs& a, int64_t blk, Acc<NT>& ex) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const void* ra = sx_ra;
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t row = blk * BR + 16 * warp + g + 8 * (e >> 1);
        const int col = 8 * t + 2 * q + (e & 1);
        ex.v[t][e] = (a.tp_world == 0 && row < a.n && col < a.m)
                         ? load_as_f32_cg(ra, a.ra_dtype, col * a.srm + row * a.srn) : 0.f;
      }
  }
  FD_DEV static void run(const GemvArgs& a, int64_t blk, const Acc<NT>& acc, const Acc<NT>& ex, float* /*xchg*/) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    if (a.tp_world > 0) {  // tensor parallel: the fp32 partial goes to every rank's exchange buffer
      tp_publish(a, blk, acc, sx_seq);
      return;
    }
    T* y = reinterpret_cast<T*>(sx_y);
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t row = blk * BR + 16 * warp + g + 8 * (e >> 1);
        const int col = 8 * t + 2 * q + (e & 1);
        if (row < a.n && col < a.m) y[col * a.sym + row * a.syn] = from_f32<T>(acc.v[t][e] + ex.v[t][e]);
      }
  }
};

// Gate/up + SwiGLU: warps 0..3 hold gate rows, warps 4..7 the matching up rows.
// gate and up are rounded to T first, as the reference rounds gate_up
// (reference.py:390, ops.py:313), then mid = round(silu(gate) * up).
template <typename T, int NT>
struct Epilogue<T, NT, MODE_GATEUP> {
  FD_DEV static void extras(const GemvArgs&, int64_t, Acc<NT>& ex) { ex.zero(); }
  FD_DEV static void run(const GemvArgs& a, int64_t blk, const Acc<NT>& acc, const Acc<NT>& /*ex*/, float* xchg) {
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

// GATEUP_S: the same epilogue (only the activation's path differs).
template <typename T, int NT>
struct Epilogue<T, NT, MODE_GATEUP_S> : Epilogue<T, NT, MODE_GATEUP> {};

// Split-K bookkeeping.  A CTA's range [s0, s1) holds at most two blocks it
// does not cover whole: the block it starts inside (slot 0) and the block it
// ends inside (slot 1).  Their partials go to the CTA's two slots with plain
// stores as soon as each is finished; both are announced together at the end
// of the range (settle), so finishing the first one never stalls the weight
// stream.  Every block's last-arriving contributor sums the slots of all its
// contributors in CTA order -- the result does not depend on timing -- applies
// the epilogue and re-zeroes the block's counter.
template <int NT>
FD_DEV void write_slot(const GemvArgs& a, int slot, const Acc<NT>& acc, int64_t c) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  float* sp = a.slots + (c * 2 + slot) * (BR * MT_MAX);
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = 16 * warp + g + 8 * h;
      const int col = 8 * t + 2 * q;
      *reinterpret_cast<float2*>(sp + r * MT_MAX + col) = make_float2(acc.v[t][2 * h], acc.v[t][2 * h + 1]);
    }
}

// Sum block blk's partials (every contributor's slot, in CTA order) and run
// the epilogue with the addends `ex`.  Called by all consumer threads of the
// CTA that completes the block.  `own`, when given, is contributor `self`'s
// partial still in registers (its slot was never written); the sum is the
// same either way.
template <typename T, int NT, int MODE>
FD_DEV void reduce_block(const GemvArgs& a, int64_t blk, float* xchg, int64_t G, const Acc<NT>& ex,
                         const Acc<NT>* own = nullptr, int64_t self = -1) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t cf = cta_of(blk * a.ks, a.total, G);
  const int64_t cl = cta_of((blk + 1) * a.ks - 1, a.total, G);
  Acc<NT> sum;
  sum.zero();
  // Contributors' slots are loaded UNROLL at a time, all in flight together
  // (one L2 round trip per batch, not one per slot), then added in CTA order.
  constexpr int UNROLL = 8;
  for (int64_t c0 = cf; c0 <= cl; c0 += UNROLL) {
    float2 v[UNROLL][NT][2];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int64_t cc = c0 + u;
      const bool mine = own != nullptr && cc == self;
      const int sl = (cc <= cl && blk != range_start(cc, a.total, G) / a.ks) ? 1 : 0;
      const float* rp = a.slots + (cc * 2 + sl) * (BR * MT_MAX);
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          v[u][t][h] = mine ? make_float2(own->v[t][2 * h], own->v[t][2 * h + 1])
                       : cc <= cl ? __ldcg(reinterpret_cast<const float2*>(rp + (16 * warp + g + 8 * h) * MT_MAX +
                                                                            8 * t + 2 * q))
                                  : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          sum.v[t][2 * h] += v[u][t][h].x;
          sum.v[t][2 * h + 1] += v[u][t][h].y;
        }
  }
  Epilogue<T, NT, MODE>::run(a, blk, sum, ex, xchg);
  if (threadIdx.x == 0) a.counters[blk] = 0;
}

// reduce_block for the head of its final block when every other contributor
// has published and their partials are staged in shared memory (`fin`): the
// same sum, in the same order -- 0 + own + each later contributor in CTA
// order, then + 0 for reduce_block's unused batch entries (x + 0 turns -0
// into +0, so it stays) -- hence the same bits.
template <typename T, int NT, int MODE>
FD_DEV void reduce_staged(const GemvArgs& a, int64_t blk, const float* fin, float* xchg, int64_t G,
                          const Acc<NT>& ex, const Acc<NT>& own, int64_t c) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int others = static_cast<int>(cta_of((blk + 1) * a.ks - 1, a.total, G) - c);
  Acc<NT> sum;
  sum.zero();
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) sum.v[t][e] += own.v[t][e];
  for (int o = 1; o <= others; ++o) {
    const float* sp = fin + (o - 1) * (BR * 8 * NT);
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float2 v = *reinterpret_cast<const float2*>(sp + (16 * warp + g + 8 * h) * 8 * NT + 8 * t + 2 * q);
        sum.v[t][2 * h] += v.x;
        sum.v[t][2 * h + 1] += v.y;
      }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) sum.v[t][e] += 0.f;
  Epilogue<T, NT, MODE>::run(a, blk, sum, ex, xchg);
  if (threadIdx.x == 0) a.counters[blk] = 0;
}

// Publish the partial of block blk (already in this CTA's slot) and, if this
// CTA is the block's last contributor, reduce it.  All consumer threads.
template <typename T, int NT, int MODE>
FD_DEV void settle(const GemvArgs& a, int64_t blk, float* xchg, int64_t G, int* s_last) {
  Acc<NT> ex;
  Epilogue<T, NT, MODE>::extras(a, blk, ex);  // in flight during the bookkeeping below
  __threadfence();  // this thread's slot stores are visible device-wide ...
  consumer_sync();  // ... for every consumer thread, before the count below
  if (threadIdx.x == 0) {
    const int64_t cf = cta_of(blk * a.ks, a.total, G);
    const int64_t cl = cta_of((blk + 1) * a.ks - 1, a.total, G);
    *s_last = atomicAdd(a.counters + blk, 1) == static_cast<int>(cl - cf);
  }
  consumer_sync();
  if (*s_last) {
    __threadfence();
    reduce_block<T, NT, MODE>(a, blk, xchg, G, ex);
  }
}


// The first block of a CTA's range, when the CTA does not cover all of it and
// the block ends before the range does, is finished mid-stream.  Its partial
// is written to slot 0 and published by a separate announcer warp (fence +
// counter), so the consumer warps go on streaming instead of waiting through
// those memory round trips; if the announcer finds this CTA completed the
// block, the consumers reduce it at the end of their range.
// One kernel may run several phases: `parity` is the phase of the two
// mbarriers for this phase's hand-off (they complete once per phase that has
// a mid block), and the flags carry `tag` (unique per phase, never 0) rather
// than 1, so no flag needs resetting between phases.
struct MidSync {
  uint64_t* ready;  // consumer warps -> announcer: slot 0 written (count GW)
  uint64_t* done;   // announcer -> consumers: published, *last valid (count 1)
  int* last;
  int* fast;        // announcer -> consumers: every other contributor of the final block has published
  int* decided;     // consumers -> announcer: the final block's path is chosen, stop watching
  uint32_t parity;
  int tag;
};

// This CTA holds the first step of its final block but not the whole block:
// the other contributors (later CTAs) process their parts at the start of
// their ranges, so they have usually published before this CTA gets there.
FD_DEV bool head_of_final(int64_t s0, int64_t s1, int64_t ks) {
  if (s1 <= s0) return false;  // an empty range (a CTA past a phase's grid) has no final block
  const int64_t bf = (s1 - 1) / ks;
  return s0 <= bf * ks && s1 < (bf + 1) * ks;
}

// Lane 0 of the announcer warp: watch the final block's count until every
// other contributor has published (then tell the consumers they may finish
// the block straight from their registers) or the consumers have decided.
FD_DEV void watch_final(const GemvArgs& a, const MidSync& ms, int64_t s0, int64_t s1, int64_t G, int64_t c) {
  if (!head_of_final(s0, s1, a.ks)) return;
  const int64_t bf = (s1 - 1) / a.ks;
  const int others = static_cast<int>(cta_of((bf + 1) * a.ks - 1, a.total, G) - c);
  const uint64_t t0 = globaltimer();
  while (*reinterpret_cast<volatile int*>(ms.decided) != ms.tag) {
    if (ld_acquire_gpu(a.counters + bf) == others) {
      *reinterpret_cast<volatile int*>(ms.fast) = ms.tag;
      return;
    }
    if (globaltimer() - t0 > kWaitNs) return;
    __nanosleep(1000);  // a light poll: the answer is only needed at the end of the range
  }
}

// The final block's later contributors publish at the start of their ranges,
// long before the head reaches its last step, yet reading their partials
// from L2 there (behind a fence, with HBM saturated) costs about 2 us at the
// end of most ranges -- the kernel's critical tail.  So, where the launch
// reserved the room (GemvArgs::fin_stage), the announcer warp copies them
// into shared memory as soon as they are published: at most kFinOthers
// contributors, the 8 * NT columns of each row that the MMA fragments hold.
constexpr int kFinOthers = 2;
__host__ __device__ inline size_t fin_stage_bytes(int nt) {
  return static_cast<size_t>(kFinOthers) * BR * 8 * nt * sizeof(float);
}
// Whether the final block of range [s0, s1) of CTA c is served from staged
// partials.  Batches up to 8 rows (one 8-column MMA tile, NT = 1) only: the
// 16-row kernels have no registers to spare for the staging code.
template <int NT>
FD_DEV bool fin_staged(const GemvArgs& a, int64_t s1, int64_t G, int64_t c) {
  if (NT != 1 || !a.fin_stage) return false;
  const int64_t bf = (s1 - 1) / a.ks;
  return cta_of((bf + 1) * a.ks - 1, a.total, G) - c <= kFinOthers;
}

// watch_final for the whole announcer warp (lane 0 polls), staging the other
// contributors' partials into `fin` before raising the flag when fin_staged.
template <int NT>
FD_DEV void watch_final_staged(const GemvArgs& a, const MidSync& ms, int64_t s0, int64_t s1, int64_t G, int64_t c,
                               float* fin) {
  if (!head_of_final(s0, s1, a.ks)) return;
  const int lane = threadIdx.x & 31;
  const int64_t bf = (s1 - 1) / a.ks;
  const int others = static_cast<int>(cta_of((bf + 1) * a.ks - 1, a.total, G) - c);
  const uint64_t t0 = globaltimer();
  int state = 0;  // 1: every other contributor has published; 2: stop watching
  while (true) {
    if (lane == 0) {
      if (*reinterpret_cast<volatile int*>(ms.decided) == ms.tag || globaltimer() - t0 > kWaitNs)
        state = 2;
      else if (ld_acquire_gpu(a.counters + bf) == others)
        state = 1;
    }
    state = __shfl_sync(0xffffffffu, state, 0);
    if (state != 0) break;
    __nanosleep(1000);  // a light poll: the answer is only needed at the end of the range
  }
  if (state == 2) return;
  __syncwarp();  // lane 0's acquire of the count orders every lane's slot reads after it
  if (fin_staged<NT>(a, s1, G, c)) {
    constexpr int V = 2 * NT;             // float4 per row
    constexpr int PER = BR * V / 32;      // float4 per lane per contributor
    for (int o = 1; o <= others; ++o) {
      const int64_t cc = c + o;
      const int sl = bf != range_start(cc, a.total, G) / a.ks ? 1 : 0;
      const float* rp = a.slots + (cc * 2 + sl) * (BR * MT_MAX);
      float* dst = fin + (o - 1) * (BR * 8 * NT);
      constexpr int CH = 8;  // float4 in flight per lane (registers: the consumers' budget is tight)
#pragma unroll
      for (int u0 = 0; u0 < PER; u0 += CH) {
        float4 v[CH];
#pragma unroll
        for (int u = 0; u < CH; ++u) {
          const int idx = lane + 32 * (u0 + u);
          v[u] = __ldcg(reinterpret_cast<const float4*>(rp + (idx / V) * MT_MAX) + idx % V);
        }
#pragma unroll
        for (int u = 0; u < CH; ++u) {
          const int idx = lane + 32 * (u0 + u);
          reinterpret_cast<float4*>(dst + (idx / V) * 8 * NT)[idx % V] = v[u];
        }
      }
    }
    __syncwarp();
    __threadfence_block();  // the staged partials before the flag
  }
  if (lane == 0) *reinterpret_cast<volatile int*>(ms.fast) = ms.tag;
}

FD_DEV bool has_mid_block(int64_t s0, int64_t s1, int64_t ks) { return s0 % ks != 0 && (s0 / ks + 1) * ks < s1; }

// Lane 0 of the announcer warp.
FD_DEV void announce_mid(const GemvArgs& a, const MidSync& ms, int64_t s0, int64_t s1, int64_t G, int* s_abort) {
  if (!has_mid_block(s0, s1, a.ks)) return;
  const int64_t b0 = s0 / a.ks;
  int last = 0;
  if (mbar_wait(ms.ready, ms.parity)) {
    if (!*reinterpret_cast<volatile int*>(s_abort)) {
      __threadfence();  // the consumers' slot stores (ordered before the mbarrier) first
      const int64_t cf = cta_of(b0 * a.ks, a.total, G);
      const int64_t cl = cta_of((b0 + 1) * a.ks - 1, a.total, G);
      last = atomicAdd(a.counters + b0, 1) == static_cast<int>(cl - cf);
    }
  } else {
    atomicOr(a.status, kStatusFullTimeout);
    *s_abort = 1;
  }
  *ms.last = last;
  mbar_arrive(ms.done);
}

// ------------------------------------------------------------ the ring
// Shared-memory layout (1024-byte aligned base):
//   [W ring: S x B x 16 KB][X region][xchg: 64 x 16 floats][full[12]][empty[12]]
//   [fin: GATEUP launches with fin_stage, kFinOthers x BR x 8 * NT floats]
// X region: LINEAR and GATEUP_S activation boxes (S x B x x_slot), or the
// GATEUP normalised batch (ks x B chunks of [m x 128 B]).
struct Ring {
  unsigned char* wst;
  unsigned char* xreg;
  float* xchg;
  uint64_t* full;
  uint64_t* empty;
  float* fin;  // GATEUP with fin_stage: [kFinOthers][BR][8 * NT] staged partials
  int S, B, x_slot;
  int64_t w_stage;
};

FD_DEV Ring carve_ring(unsigned char* smem_raw, int S, int B, int x_slot, int64_t x_bytes) {
  Ring r;
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~static_cast<uintptr_t>(1023));
  r.S = S;
  r.B = B;
  r.x_slot = x_slot;
  r.w_stage = static_cast<int64_t>(B) * BOX_BYTES;
  r.wst = smem;
  r.xreg = smem + S * r.w_stage;
  r.xchg = reinterpret_cast<float*>(r.xreg + ((x_bytes + 15) & ~15ll));
  r.full = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(r.xchg) + (BR / 2) * MT_MAX * 4);
  r.empty = r.full + MAX_STAGES;
  r.fin = reinterpret_cast<float*>(r.empty + MAX_STAGES);
  return r;
}

FD_DEV void ring_init(const Ring& r) {
  for (int i = 0; i < r.S; ++i) {
    mbar_init(&r.full[i], 1);
    mbar_init(&r.empty[i], GW);
  }
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

template <int MODE>
FD_DEV uint32_t stage_bytes(const Ring& r, const GemvArgs& a) {
  return static_cast<uint32_t>(r.w_stage) + (streams_x(MODE) ? static_cast<uint32_t>(r.B * a.m * 128) : 0u);
}

// Weight boxes of phase step t into ring index gi.
template <int MODE>
FD_DEV void issue_w(const Ring& r, const CUtensorMap* map, const GemvArgs& a, int64_t t, int64_t gi, uint64_t pol) {
  const int64_t b = t / a.ks, kk = t - b * a.ks;
  const int s = static_cast<int>(gi % r.S);
  unsigned char* dst = r.wst + s * r.w_stage;
  for (int j = 0; j < r.B; ++j) {
    const int32_t col = static_cast<int32_t>((kk * r.B + j) * KC);
    if (gateup_mode(MODE))
      tma_load_3d(dst + j * BOX_BYTES, map, col, static_cast<int32_t>(b * (BR / 2)), 0, &r.full[s], pol);
    else
      tma_load_2d(dst + j * BOX_BYTES, map, col, static_cast<int32_t>(b * BR), &r.full[s], pol);
  }
}
// Activation boxes (LINEAR) of phase step t into ring index gi.
FD_DEV void issue_x(const Ring& r, const CUtensorMap* xmap, const GemvArgs& a, int64_t t, int64_t gi) {
  const int64_t kk = t - (t / a.ks) * a.ks;
  const int s = static_cast<int>(gi % r.S);
  for (int j = 0; j < r.B; ++j)
    tma_load_2d_plain(r.xreg + (s * r.B + j) * r.x_slot, xmap, static_cast<int32_t>((kk * r.B + j) * KC), 0,
                      &r.full[s]);
}

// Producer p's share of one phase: phase steps [s0, s1) occupy ring indices
// base .. base + (s1 - s0).  For a LINEAR phase the activation may be written
// by whatever ran before: the weight boxes of the phase's first S steps go out
// first, then `ready()` (a bounded wait) makes the activation readable, then
// their activation boxes follow.  Returns false when a wait expired.
template <int MODE, typename Ready>
FD_DEV bool produce_phase(const Ring& r, const CUtensorMap* wmap, const CUtensorMap* xmap, const GemvArgs& a,
                          int64_t s0, int64_t s1, int64_t base, int p, int P, uint64_t pol, int* s_abort,
                          Ready ready) {
  const int64_t n = s1 - s0;
  const uint32_t sb = stage_bytes<MODE>(r, a);
  const int64_t npre = n < r.S ? n : r.S;
  // first index of this producer at or after `base`
  int64_t first = base + ((p - base % P) % P + P) % P;
  auto acquire = [&](int64_t gi) -> bool {  // stage of ring index gi is free again
    if (gi < r.S) return true;
    const int s = static_cast<int>(gi % r.S);
    if (!mbar_wait(&r.empty[s], static_cast<uint32_t>((gi / r.S - 1) & 1))) {
      atomicOr(a.status, kStatusEmptyTimeout);
      *s_abort = 1;
      return false;
    }
    return !*reinterpret_cast<volatile int*>(s_abort);
  };
  int64_t gi = first;
  for (; gi < base + npre; gi += P) {
    if (!acquire(gi)) return false;
    mbar_expect_tx(&r.full[gi % r.S], sb);
    issue_w<MODE>(r, wmap, a, s0 + (gi - base), gi, pol);
  }
  if (streams_x(MODE)) {
    if (!ready()) return false;
    for (int64_t g2 = first; g2 < base + npre; g2 += P) issue_x(r, xmap, a, s0 + (g2 - base), g2);
  }
  for (; gi < base + n; gi += P) {
    if (!acquire(gi)) return false;
    mbar_expect_tx(&r.full[gi % r.S], sb);
    issue_w<MODE>(r, wmap, a, s0 + (gi - base), gi, pol);
    if (streams_x(MODE)) issue_x(r, xmap, a, s0 + (gi - base), gi);
  }
  return true;
}

// Producer p: wait until every copy it issued to the last S ring indices
// [end - S, end) has landed (their stages are never refilled, so the phase
// parity is unambiguous).  Keeps the CTA alive while copies are in flight.
FD_DEV void producer_drain(const Ring& r, int64_t end, int p, int P) {
  const int64_t lo = end > r.S ? end - r.S : 0;
  for (int64_t gi = lo + ((p - lo % P) % P + P) % P; gi < end; gi += P)
    if (!mbar_wait(&r.full[gi % r.S], static_cast<uint32_t>((gi / r.S) & 1))) break;
}

// RMSNorm of the m hidden rows into the GATEUP X region, rounded to T
// (reference.py:389 rounds `normed` to the activation dtype), stored as
// 64-column chunks of [m x 128 B] with the same swizzle as a TMA tile;
// columns past k (to the end of the last step) are zero.  The norm weight
// (k elements of norm_dtype) is in shared memory at `nw`, copied there by a
// bulk TMA load that completes on `nw_bar`.  Called by all consumer threads;
// ends with a consumer barrier.
//
// Every CTA normalises the whole batch between the launch (or the phase
// barrier) and its first tensor-core step, so this latency- and issue-bound
// SIMT work sits on the critical path (measured alone on one B200 SM at
// k = 4096: about 1,800 cycles at m = 1 and 5,700 at m = 8).  The steps:
//   1. cp.async (through L2: rows written earlier in the same kernel are
//      read coherently) of every 16-byte vector of every row straight to its
//      final place in X -- one round trip for the whole batch;
//   2. each thread's sums of squares over the vectors it copied (readable by
//      that thread after its own wait), RB rows at a time so that their
//      shared loads, FMAs and warp butterflies overlap;
//   3. one thread per row adds the warps' sums (in warp order) and stores
//      the row's scale rsqrt(mean + eps) -- all rows at once;
//   4. the scale in place, RB rows per norm-weight vector (loaded once):
//      (x * scale) * w, rounded to T.
// The fp32 products go through packed f32x2 multiplies (sm_100): each lane
// rounds like the scalar multiply, so the bits are those of x * scale * w.
// Sum order is fixed (even and odd columns of a thread's vectors as two
// running FMA sums, then lanes by butterfly, then warps in index order), so
// results are run-to-run exact.
FD_DEV uint64_t f32x2_of(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
FD_DEV float2 f32x2_split(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
FD_DEV uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
FD_DEV uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// one 32-bit word of two T elements -> {lo, hi} as f32x2 (exact)
template <typename T>
FD_DEV uint64_t pair_f32x2(uint32_t w) {
  const float2 f = unpack2<T>(w);
  return f32x2_of(f.x, f.y);
}
// 8 norm-weight elements of a runtime dtype at p (shared memory) as 4 f32x2 pairs
FD_DEV void nw_pairs(const unsigned char* p, int dtype, uint64_t* w) {
  if (dtype == FD_F32) {
    const uint4 lo = *reinterpret_cast<const uint4*>(p), hi = *reinterpret_cast<const uint4*>(p + 16);
    w[0] = (static_cast<uint64_t>(lo.y) << 32) | lo.x;
    w[1] = (static_cast<uint64_t>(lo.w) << 32) | lo.z;
    w[2] = (static_cast<uint64_t>(hi.y) << 32) | hi.x;
    w[3] = (static_cast<uint64_t>(hi.w) << 32) | hi.z;
  } else {
    const uint4 r = *reinterpret_cast<const uint4*>(p);
    if (dtype == FD_BF16) {
      w[0] = pair_f32x2<__nv_bfloat16>(r.x); w[1] = pair_f32x2<__nv_bfloat16>(r.y);
      w[2] = pair_f32x2<__nv_bfloat16>(r.z); w[3] = pair_f32x2<__nv_bfloat16>(r.w);
    } else {
      w[0] = pair_f32x2<__half>(r.x); w[1] = pair_f32x2<__half>(r.y);
      w[2] = pair_f32x2<__half>(r.z); w[3] = pair_f32x2<__half>(r.w);
    }
  }
}
FD_DEV uint4 ld_shared16(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_addr(p))
               : "memory");
  return v;
}
FD_DEV void cp_async16_cg(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
FD_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// byte offset of row mrow's 16-byte vector v in the GATEUP X region of m rows
FD_DEV int gateup_x_off(int m, int mrow, int v) { return ((v >> 3) * m + mrow) * 128 + (((v & 7) ^ (mrow & 7)) << 4); }

template <typename T, int RB>
FD_DEV void norm_rows(const GemvArgs& a, const void* hidden, const Ring& r, float (*s_sumsq)[MT_MAX],
                      const unsigned char* nw, uint64_t* nw_bar, uint32_t nw_parity) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m = a.m;
  const int nvec = static_cast<int>(a.k / 8);
  const int nvec_pad = static_cast<int>(a.ks * r.B * (KC / 8));
  unsigned char* xs = r.xreg;
  const T* hb = reinterpret_cast<const T*>(hidden);
  // 1. every vector of every row to its place in X (zeros past k)
#pragma unroll 1
  for (int v = tid; v < nvec_pad; v += CONSUMERS) {
    if (v < nvec) {
#pragma unroll 4
      for (int mrow = 0; mrow < m; ++mrow)
        cp_async16_cg(xs + gateup_x_off(m, mrow, v), reinterpret_cast<const uint4*>(hb + mrow * a.hidden_stride) + v);
    } else {
      for (int mrow = 0; mrow < m; ++mrow) st_shared16(xs + gateup_x_off(m, mrow, v), make_uint4(0, 0, 0, 0));
    }
  }
  cp_async_wait_all();
  // 2. sums of squares, RB rows at a time
#pragma unroll 1
  for (int r0 = 0; r0 < m; r0 += RB) {
    uint64_t acc[RB];
#pragma unroll
    for (int q = 0; q < RB; ++q) acc[q] = 0;  // {+0.f, +0.f}
#pragma unroll 1
    for (int v = tid; v < nvec; v += CONSUMERS) {
      uint4 raw[RB];
#pragma unroll
      for (int q = 0; q < RB; ++q)
        if (RB == 1 || r0 + q < m) raw[q] = ld_shared16(xs + gateup_x_off(m, r0 + q, v));
#pragma unroll
      for (int q = 0; q < RB; ++q) {
        if (RB == 1 || r0 + q < m) {
          const uint64_t p0 = pair_f32x2<T>(raw[q].x), p1 = pair_f32x2<T>(raw[q].y);
          const uint64_t p2 = pair_f32x2<T>(raw[q].z), p3 = pair_f32x2<T>(raw[q].w);
          acc[q] = fma_f32x2(p0, p0, acc[q]);
          acc[q] = fma_f32x2(p1, p1, acc[q]);
          acc[q] = fma_f32x2(p2, p2, acc[q]);
          acc[q] = fma_f32x2(p3, p3, acc[q]);
        }
      }
    }
    float t[RB];
#pragma unroll
    for (int q = 0; q < RB; ++q) {
      const float2 h = f32x2_split(acc[q]);
      t[q] = h.x + h.y;
    }
#pragma unroll
    for (int q = 0; q < RB; ++q) t[q] = warp_sum(t[q]);
    if (lane == 0) {
#pragma unroll
      for (int q = 0; q < RB; ++q)
        if (RB == 1 || r0 + q < m) s_sumsq[warp][r0 + q] = t[q];
    }
  }
  consumer_sync();
  // 3. the rows' scales (row i by thread i; it alone reads column i)
  if (tid < m) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < GW; ++w) tot += s_sumsq[w][tid];
    s_sumsq[0][tid] = rsqrtf(tot / static_cast<float>(a.k) + a.eps);
  }
  if (!mbar_wait(nw_bar, nw_parity)) atomicOr(a.status, kStatusFullTimeout);
  consumer_sync();
  // 4. scale in place
  const int wes = a.norm_dtype == FD_F32 ? 4 : 2;
#pragma unroll 1
  for (int v = tid; v < nvec; v += CONSUMERS) {
    uint64_t w[4];
    nw_pairs(nw + static_cast<int64_t>(v) * 8 * wes, a.norm_dtype, w);
#pragma unroll 1
    for (int r0 = 0; r0 < m; r0 += RB) {
      uint4 raw[RB];
#pragma unroll
      for (int q = 0; q < RB; ++q)
        if (RB == 1 || r0 + q < m) raw[q] = ld_shared16(xs + gateup_x_off(m, r0 + q, v));
#pragma unroll
      for (int q = 0; q < RB; ++q) {
        if (RB == 1 || r0 + q < m) {
          const float inv = s_sumsq[0][r0 + q];
          const uint64_t i2 = f32x2_of(inv, inv);
          const float2 o0 = f32x2_split(mul_f32x2(mul_f32x2(pair_f32x2<T>(raw[q].x), i2), w[0]));
          const float2 o1 = f32x2_split(mul_f32x2(mul_f32x2(pair_f32x2<T>(raw[q].y), i2), w[1]));
          const float2 o2 = f32x2_split(mul_f32x2(mul_f32x2(pair_f32x2<T>(raw[q].z), i2), w[2]));
          const float2 o3 = f32x2_split(mul_f32x2(mul_f32x2(pair_f32x2<T>(raw[q].w), i2), w[3]));
          uint4 packed;
          packed.x = pack2<T>(o0.x, o0.y);
          packed.y = pack2<T>(o1.x, o1.y);
          packed.z = pack2<T>(o2.x, o2.y);
          packed.w = pack2<T>(o3.x, o3.y);
          st_shared16(xs + gateup_x_off(m, r0 + q, v), packed);
        }
      }
    }
  }
  consumer_sync();
}

// `hidden`: the rows to normalise (a.hidden for a single launch; the stack
// passes each layer's input).  The row block RB is the batch rounded up to
// 1, 2, 4 or 8, at most RBMAX (larger batches take several blocks): a kernel
// whose consumer warps hold more state across the prologue (the persistent
// stack) takes a smaller block rather than spill.
template <typename T, int RBMAX = 8>
FD_DEV void norm_to_smem(const GemvArgs& a, const void* hidden, const Ring& r, float (*s_sumsq)[MT_MAX],
                         const unsigned char* nw, uint64_t* nw_bar, uint32_t nw_parity = 0) {
  if (a.m == 1 || RBMAX == 1)
    norm_rows<T, 1>(a, hidden, r, s_sumsq, nw, nw_bar, nw_parity);
  else if (a.m == 2 || RBMAX == 2)
    norm_rows<T, 2>(a, hidden, r, s_sumsq, nw, nw_bar, nw_parity);
  else if (a.m <= 4 || RBMAX == 4)
    norm_rows<T, (RBMAX < 4 ? RBMAX : 4)>(a, hidden, r, s_sumsq, nw, nw_bar, nw_parity);
  else
    norm_rows<T, (RBMAX < 8 ? RBMAX : 8)>(a, hidden, r, s_sumsq, nw, nw_bar, nw_parity);
}

// Consumer warps' share of one phase: phase steps [s0, s1) at ring indices
// base ..; flushes every finished block.  Returns false when a wait expired.
// cl_out: the cluster split (gemv_cluster_kernel) -- the range lies inside
// one block and its partial is returned here for the cluster's reduction
// instead of going through the split-K slots.
template <typename T, int NT, int KIND, int MP, int MODE>
FD_DEV bool consume_phase(const GemvArgs& a, const Ring& r, int64_t s0, int64_t s1, int64_t base, int64_t G,
                          int64_t c, int* s_last, int* s_abort, const MidSync& ms, Acc<NT>* cl_out = nullptr) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int B = r.B;
  Acc<NT> acc;
  acc.zero();
  float sacc[2][MP];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr)
#pragma unroll
    for (int mm = 0; mm < MP; ++mm) sacc[rr][mm] = 0.f;

  const int r0 = 16 * warp + g;  // weight rows of this lane in every box: r0, r0 + 8
  int64_t cb = s0 / a.ks, ck = s0 - (s0 / a.ks) * a.ks;
  for (int64_t it = 0; it < s1 - s0; ++it) {
    const int64_t gi = base + it;
    const int s = static_cast<int>(gi % r.S);
    if (!mbar_wait(&r.full[s], static_cast<uint32_t>((gi / r.S) & 1))) {
      atomicOr(a.status, kStatusFullTimeout);
      *s_abort = 1;
      return false;  // every consumer warp times out on this same stage
    }
    uint4 wa[MAX_BOXES][2], wb[MAX_BOXES][2];
#pragma unroll
    for (int j = 0; j < MAX_BOXES; ++j) {
      if (j < B) {
        const unsigned char* wt = r.wst + s * r.w_stage + j * BOX_BYTES;
        wa[j][0] = *reinterpret_cast<const uint4*>(wt + swz(r0, 2 * q));
        wa[j][1] = *reinterpret_cast<const uint4*>(wt + swz(r0, 2 * q + 1));
        wb[j][0] = *reinterpret_cast<const uint4*>(wt + swz(r0 + 8, 2 * q));
        wb[j][1] = *reinterpret_cast<const uint4*>(wt + swz(r0 + 8, 2 * q + 1));
      }
    }
    // activation box j of this step: [m rows x 128 B] (swizzled by row & 7)
    auto xbox = [&](int j) -> const unsigned char* {
      if (streams_x(MODE)) return r.xreg + (s * B + j) * r.x_slot;
      if (MODE == MODE_LINEAR_X) return r.xreg + ((it * B + j) * a.m) * 128;
      return r.xreg + ((ck * B + j) * a.m) * 128;
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
      if (lane == 0) mbar_arrive(&r.empty[s]);
      // physical column 16q + 4h + j  <->  logical k of MMA h: (2q, 2q+1, 2q+8, 2q+9)
      // The step's products are summed by the MMAs into a fresh accumulator,
      // which is then added to the running sum with an fp32 add: an MMA adds
      // its products into C with truncating alignment, so over K = 14336..28672
      // a running C would lose low bits at every one of K/16 MMAs.
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        float st[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < MAX_BOXES; ++j) {
          if (j < B) {
            mma16816<T>(st, wa[j][0].x, wb[j][0].x, wa[j][0].y, wb[j][0].y, xa[j][t][0].x, xa[j][t][0].y);
            mma16816<T>(st, wa[j][0].z, wb[j][0].z, wa[j][0].w, wb[j][0].w, xa[j][t][0].z, xa[j][t][0].w);
            mma16816<T>(st, wa[j][1].x, wb[j][1].x, wa[j][1].y, wb[j][1].y, xa[j][t][1].x, xa[j][t][1].y);
            mma16816<T>(st, wa[j][1].z, wb[j][1].z, wa[j][1].w, wb[j][1].w, xa[j][t][1].z, xa[j][t][1].w);
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) acc.v[t][e] += st[e];
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
      if (lane == 0) mbar_arrive(&r.empty[s]);
    }
    // ---- block finished (or range ends): flush
    ++ck;
    if (ck == a.ks || it + 1 == s1 - s0) {
      if (KIND == 1) {
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
#pragma unroll
          for (int mm = 0; mm < MP; ++mm) {
            float v = sacc[rr][mm];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            sacc[rr][mm] = v;
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
      const bool covered = (s0 <= cb * a.ks) && (s1 >= (cb + 1) * a.ks);
      if (cl_out) {
        *cl_out = acc;  // the range's one flush: the cluster reduces it
      } else if (covered) {
        Acc<NT> ex;
        Epilogue<T, NT, MODE>::extras(a, cb, ex);
        Epilogue<T, NT, MODE>::run(a, cb, acc, ex, r.xchg);
      } else if (it + 1 < s1 - s0) {
        // the range's first block ends mid-stream: hand it to the announcer
        write_slot<NT>(a, 0, acc, c);
        __syncwarp();
        if (lane == 0) mbar_arrive(ms.ready);
      } else if (gateup_mode(MODE) && head_of_final(s0, s1, a.ks)) {
        Acc<NT> ex;
        Epilogue<T, NT, MODE>::extras(a, cb, ex);
        if (threadIdx.x == 0) {
          *s_last = *reinterpret_cast<volatile int*>(ms.fast) == ms.tag;
          *reinterpret_cast<volatile int*>(ms.decided) = ms.tag;
          __threadfence_block();  // the flag before the staged partials
        }
        consumer_sync();
        if (*s_last) {
          // every other contributor has published: this CTA completes the
          // block without publishing its own partial
          if (fin_staged<NT>(a, s1, G, c)) {
            reduce_staged<T, NT, MODE>(a, cb, r.fin, r.xchg, G, ex, acc, c);
          } else {
            __threadfence();
            reduce_block<T, NT, MODE>(a, cb, r.xchg, G, ex, &acc, c);
          }
        } else {
          write_slot<NT>(a, cb == s0 / a.ks ? 0 : 1, acc, c);
          settle<T, NT, MODE>(a, cb, r.xchg, G, s_last);
        }
      } else {
        write_slot<NT>(a, cb == s0 / a.ks ? 0 : 1, acc, c);
        settle<T, NT, MODE>(a, cb, r.xchg, G, s_last);
      }
      acc.zero();
#pragma unroll
      for (int rr = 0; rr < 2; ++rr)
#pragma unroll
        for (int mm = 0; mm < MP; ++mm) sacc[rr][mm] = 0.f;
      ck = 0;
      ++cb;
    }
  }
  if (has_mid_block(s0, s1, a.ks)) {
    if (!mbar_wait(ms.done, ms.parity)) {
      atomicOr(a.status, kStatusFullTimeout);
      *s_abort = 1;
      return false;
    }
    if (*ms.last) {
      Acc<NT> ex;
      Epilogue<T, NT, MODE>::extras(a, s0 / a.ks, ex);
      __threadfence();
      reduce_block<T, NT, MODE>(a, s0 / a.ks, r.xchg, G, ex);
    }
  }
  return true;
}

// ------------------------------------------------------------ host side
inline size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

constexpr int kMaxCtasPerSm = 2;  // workspace slots are sized for up to two CTAs per SM
inline int64_t max_grid() { return static_cast<int64_t>(fd_host::sm_count()) * kMaxCtasPerSm; }

// Workspace layout (fixed for a device, whatever the shape, so one buffer can
// serve every launch):  [slots: max grid x 2 x BR x MT_MAX floats]
//                       [counters: kMaxCounters ints][status word, padded to 256 B]
//                       [MLP intermediates]
inline size_t slots_bytes() { return align256(static_cast<size_t>(max_grid()) * 2 * BR * MT_MAX * sizeof(float)); }
inline size_t counters_offset() { return slots_bytes(); }
inline size_t status_offset() { return counters_offset() + kMaxCounters * sizeof(int); }
inline size_t streamk_ws_bytes() { return status_offset() + 256; }

struct Workspace {
  float* slots;
  int* counters;
  int* status;
  char* tail;
};
inline Workspace carve(void* ws) {
  char* p = static_cast<char*>(ws);
  return {reinterpret_cast<float*>(p), reinterpret_cast<int*>(p + counters_offset()),
          reinterpret_cast<int*>(p + status_offset()), p + streamk_ws_bytes()};
}

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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
inline bool make_map(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
                     const cuuint64_t* strides, const cuuint32_t* box) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, rank, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// [rows, cols] matrix with row stride `stride` elements, boxes of [box_rows x 64].
inline bool make_map_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t stride,
                        int box_rows) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(KC), static_cast<cuuint32_t>(box_rows)};
  return make_map(map, base, 2, dims, strides, box);
}

// w_gate_up [2i, h] (row stride s) as a 3-D [2][i][h] map: one [2 x 64 x 64]
// box is 64 gate rows over the matching 64 up rows.
inline bool make_gate_up_map(CUtensorMap* map, const void* w_gate_up, int64_t h, int64_t i, int64_t s) {
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(h), static_cast<cuuint64_t>(i), 2};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(s) * 2, static_cast<cuuint64_t>(i) * s * 2};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(KC), BR / 2, 2};
  return make_map(map, w_gate_up, 3, dims, strides, box);
}

__host__ __device__ inline int x_slot_bytes(int m) { return m <= 8 ? 1024 : 2048; }

__host__ __device__ inline size_t gateup_x_bytes(int m, int64_t ks, int boxes) {
  return static_cast<size_t>(ks) * boxes * m * 128;
}
__host__ __device__ inline size_t nw_copy_bytes(int64_t k, int norm_es) {
  return (static_cast<size_t>(k) * norm_es + 15) & ~static_cast<size_t>(15);
}
// The gate/up X region: the normalised batch, then the norm weight's copy.
__host__ __device__ inline size_t gateup_region_bytes(int m, int64_t ks, int boxes, int64_t k, int norm_es) {
  return gateup_x_bytes(m, ks, boxes) + nw_copy_bytes(k, norm_es);
}
__host__ __device__ inline size_t linear_x_bytes(int m, int stages, int boxes) {
  return static_cast<size_t>(stages) * boxes * x_slot_bytes(m);
}

inline size_t ring_smem_bytes(size_t xbytes, int stages, int boxes) {
  return 1024 + static_cast<size_t>(stages) * boxes * BOX_BYTES + ((xbytes + 15) & ~static_cast<size_t>(15)) +
         (BR / 2) * MT_MAX * 4 + 2 * MAX_STAGES * 8;
}

constexpr size_t kSmemPerSm = 228 * 1024;          // shared memory of one SM
constexpr size_t kSmemPerCta = 227 * 1024 - 1024;  // opt-in maximum, less static shared memory

// Pipeline geometry of one launch: producer warps, 64-column boxes per step
// and ring stages (one CTA per SM).  Measured on B200 over the Llama-3-8B MLP
// shapes (32-launch CUDA graphs, M = 1 and 8): two producer warps, 32 KB
// steps (two boxes) and four stages streamed fastest; 16 KB steps were 20-30 %
// slower, two CTAs per SM with one producer each 3-10 % slower.
// `xbytes(stages, boxes)` gives the X region the kernel needs.
struct Geometry {
  int producers, boxes, stages;
};

template <typename XBytes>
Geometry choose_geometry(XBytes xbytes) {
  Geometry g{2, 2, 4};
  bool tuned = false;
  if (const char* env = std::getenv("FD_GEMV_GEOMETRY")) {  // tuning override: "producers,boxes,stages"
    int b = 0, c = 0, d = 0;
    if (std::sscanf(env, "%d,%d,%d", &b, &c, &d) == 3 && b >= 1 && b <= MAX_PRODUCERS && c >= 1 &&
        c <= MAX_BOXES && d >= 2 && d <= MAX_STAGES) {
      g = {b, c, d};
      tuned = true;
    }
  }
  auto bytes = [&](int st) { return ring_smem_bytes(xbytes(st, g.boxes), st, g.boxes); };
  while (g.stages > 2 && bytes(g.stages) > kSmemPerCta) --g.stages;
  // By default every stage is refilled by the same producer; an override may
  // give any stage count (producers then alternate on a stage, which is
  // correct: each waits for its own index's stage to be released).
  if (!tuned) g.stages -= g.stages % g.producers;
  if (g.stages < 2 || bytes(g.stages) > kSmemPerCta) g.stages = 0;
  return g;
}

inline int from_cuda(cudaError_t e) { return e == cudaSuccess ? FD_OK : FD_ERR_LAUNCH; }

}  // namespace fd_stream

namespace fd_host {
// A post_attn_mlp stack as one persistent kernel (fd_stack.cu).  mid, ping0
// and ping1 are the workspace's intermediate buffers ([m, i], [m, h], [m, h]).
// FD_ERR_UNSUPPORTED: not served by the persistent kernel (use the chain).
int mlp_stack_persistent(const void* hidden, int32_t layers, const void* const* norm_w, int32_t norm_dtype,
                         const void* const* w_gate_up, int64_t s_gu, const void* const* w_down, int64_t s_down,
                         void* out, int32_t dtype, int32_t m, int64_t h, int64_t i, float eps, int32_t kind,
                         const fd_stream::Workspace& ws, void* mid, void* ping0, void* ping1, cudaStream_t st,
                         int32_t tp_rank = 0, int32_t tp_world = 0, void* const* exchange = nullptr,
                         int32_t tp_mmax = 0);
int mlp_stack_launches(int32_t layers, int32_t norm_dtype, int32_t m, int64_t h, int64_t i, int32_t kind);
// Kernel launches of one post_attn_mlp layer (fd_gemv.cu): gate/up (+ the
// streamed mode's norm kernel), down (+ the tensor-parallel reduce kernel).
int mlp_layer_launches(int32_t m, int64_t h, int64_t i, int32_t norm_dtype, int32_t kind, bool tensor_parallel);

// Tensor parallel: with FD_TP_FOLD=1 (and kind = dot) the rank sum runs in
// the down projection's epilogue (tp_fold_block, two launches a layer);
// otherwise in the separate tp_reduce_kernel launch (three a layer).  The
// default is the separate kernel: on 2 and 4 B200s the fold measured as fast
// or slightly slower -- it saves a launch, but each block's finishing CTA
// then holds its SM's shared memory while it waits for the peers, and the
// next layer's gate/up CTAs cannot start their weight prefetch there.
inline bool tp_fold_enabled() {
  const char* env = std::getenv("FD_TP_FOLD");
  return env && env[0] == '1';
}
}  // namespace fd_host
