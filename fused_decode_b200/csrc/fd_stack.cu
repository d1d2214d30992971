// A stack of post-attention MLP layers as ONE persistent kernel.
//
// The two-launch chain (fd_gemv.cu) pays, twice per layer, the cost of a
// kernel boundary: a grid-wide drain of the split-K tails, the next grid's
// launch, and a pipeline that refills from empty.  Here one CTA per SM runs
// every phase of every layer -- gate/up(0), down(0), gate/up(1), ... -- and
// the producer warps never stop streaming weights at a phase boundary: the
// weights do not depend on the activations, so the producers run ahead into
// the next phase as far as the ring lets them, while the consumer warps wait
// at a grid-wide barrier for the phase's input (all of the previous phase's
// blocks reduced and stored).
//
//  * Phase 2l (gate/up of layer l): the consumers RMS-normalise hidden_l into
//    shared memory (its norm weight was copied there by a bulk TMA load one
//    layer ahead) and stream w_gate_up[l]; the SwiGLU epilogue writes mid.
//  * Phase 2l+1 (down of layer l): the consumers copy the columns of mid that
//    their step range covers into shared memory, then stream w_down[l]; the
//    epilogue adds hidden_l and writes hidden_{l+1} (ping-pong buffers in the
//    workspace; the last layer writes `out`).
//  * Every phase is split stream-K over the grid exactly as a single launch
//    of the same shape is (same blocks, steps, CTA ranges and slot order), so
//    the stack's output is bit-identical to the chain's.
//  * Barrier: a counter in the workspace.  At the end of a phase each CTA's
//    consumers finish their stores and reductions, then one thread fences and
//    adds 1; phase p starts when the counter reaches p * grid.  Each CTA's
//    announcer warp, which polls every phase's count, finally waits for the
//    launch's last arrival and then adds 1 to a departure counter; the last
//    CTA to depart puts both counters back to 0 -- no CTA can still be
//    polling for an earlier count by then.  Every wait is bounded (2 s);
//    an expired wait, or an error bit another CTA set, makes the CTA leave
//    with status bit 16 set.
//  * The launch is cooperative: all CTAs are resident at once, which the
//    barrier needs.
#include "fd_stream.cuh"

#include <cstring>

using namespace fd;
using namespace fd_stream;

namespace {

constexpr int kStackMaxLayers = 32;  // per launch (kernel parameter space); longer stacks take several launches
constexpr int kStackProducers = 2;
// Warps 0-7 consume (two warpgroups); warpgroup 2 holds the two producer
// warps, the announcer warp and one idle warp.  The helpers hand registers
// back with setmaxnreg so the consumers -- which hold a step's fragments,
// the accumulators and the ring and phase state at once -- get 208 per
// thread instead of the 168 that 384 threads allow.  setmaxnreg.inc waits
// until the block's launch allotment can cover the request, so the split
// must fit it: 8*32*208 + 4*32*56 = 60416 <= 384*160, i.e. any launch
// allotment of at least 160 per thread (the build checks ptxas gives 168).
constexpr int kStackThreads = CONSUMERS + 4 * 32;
constexpr int kConsumerRegs = 208;
constexpr int kHelperRegs = 56;
static_assert(8 * 32 * kConsumerRegs + 4 * 32 * kHelperRegs <= kStackThreads * 160, "register split");
constexpr int kStatusBarrierTimeout = 16;
constexpr size_t kBarOffset = 128;  // barrier counter: inside the status area, its own 128-byte line
constexpr int kDepartOffset = 16;   // departure counter: 16 ints after the barrier counter

struct StackParams {
  CUtensorMap gu[kStackMaxLayers];  // w_gate_up[l] as [2][i][h], boxes of 64 gate over 64 up rows
  CUtensorMap dn[kStackMaxLayers];  // w_down[l] as [h][i], boxes of 128 x 64
  const void* norm_w[kStackMaxLayers];
  GemvArgs ga;  // gate/up phases: geometry and workspace (hidden, norm_w set per layer)
  GemvArgs da;  // down phases (ra, y set per layer)
  const void* hidden;
  void* out;
  char* ping[2];
  const void* mid;
  int* bar;
  char* tp_buf;     // tensor parallel: this rank's exchange buffer (its header holds the round number)
  int layers;       // layers of this launch
  int first_layer;  // index of its first layer in the whole stack
  int total_layers;
  int xact_bytes;   // activation part of the X region; the norm weight follows it
  int x_bytes;
};

FD_DEV bool phase_wait(const int* bar, int target, int* status, int* s_abort) {
  if (ld_acquire_gpu(bar) >= target) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (ld_acquire_gpu(bar) >= target) return true;
    if (*reinterpret_cast<volatile int*>(status) != 0 || *reinterpret_cast<volatile int*>(s_abort)) return false;
    if (globaltimer() - t0 > kWaitNs) {
      atomicOr(status, kStatusBarrierTimeout);
      return false;
    }
    __nanosleep(20);
  }
}

// All consumer threads: wait until `target` CTA-phases have arrived.
FD_DEV bool consumer_phase_wait(const int* bar, int target, int* status, int* s_abort) {
  if (threadIdx.x == 0 && !phase_wait(bar, target, status, s_abort)) *reinterpret_cast<volatile int*>(s_abort) = 1;
  consumer_sync();
  return !*reinterpret_cast<volatile int*>(s_abort);
}

// All consumer threads, after the phase's last store: this CTA has arrived.
FD_DEV void phase_arrive(int* bar) {
  consumer_sync();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(bar, 1);
  }
}

// All consumer threads: the columns of `src` ([m, k] rows, row stride k) that
// steps [s0, s1) of a LINEAR_X phase read, into the X region as chunks of
// [m x 128 B] in step order, swizzled like a TMA tile (the layout the
// consumers read).  Columns past k are zero.  Loads go through L2 (another
// CTA wrote them in this kernel).  Under full HBM load an L2 round trip
// takes microseconds, so each thread issues all its loads (up to U) before
// its first store: one round trip for m <= 8 at the Llama widths.
template <typename T>
FD_DEV void stage_x(const GemvArgs& a, const Ring& r, const T* src, int64_t s0, int64_t s1) {
  const int m = a.m, B = r.B;
  const int nvec = static_cast<int>((s1 - s0) * B * m * 8);
  constexpr int U = 16;
  for (int v0 = threadIdx.x; v0 < nvec; v0 += CONSUMERS * U) {
    uint4 val[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int v = v0 + u * CONSUMERS;
      val[u] = make_uint4(0, 0, 0, 0);
      if (v < nvec) {
        const int cc = v & 7, rc = v >> 3;  // rc = chunk * m + row
        const int mrow = rc % m, q = rc / m;
        const int it = q / B, j = q - it * B;
        const int64_t col = (((s0 + it) % a.ks) * B + j) * KC + cc * 8;
        if (col < a.k) val[u] = __ldcg(reinterpret_cast<const uint4*>(src + mrow * a.k + col));
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int v = v0 + u * CONSUMERS;
      if (v < nvec) {
        const int cc = v & 7, rc = v >> 3, mrow = rc % m;
        st_shared16(r.xreg + static_cast<int64_t>(rc) * 128 + ((cc ^ (mrow & 7)) << 4), val[u]);
      }
    }
  }
  consumer_sync();
}

// Tensor parallel: the reduce phase of one layer.  This CTA's share of the
// m x h outputs: wait (bounded) until every rank's tagged partial word of
// the round is in this rank's exchange buffer, sum the ranks in rank order
// (the same bits on every rank), add the residual and round.  All consumer
// threads.  False when a wait expired (status bit 8).
template <typename T>
FD_DEV bool tp_reduce_phase(const StackParams& p, int seq, const T* res, T* out, int* status) {
  const int64_t n = p.da.n;
  const int64_t total = static_cast<int64_t>(p.da.m) * n;
  const int64_t G = gridDim.x, c = blockIdx.x;
  const int64_t e1 = (c + 1) * total / G;
  const int world = p.da.tp_world;
  const int64_t rank_stride = static_cast<int64_t>(p.da.tp_mmax) * n;
  const uint2* base = reinterpret_cast<const uint2*>(p.tp_buf + p.da.tp_data_off) + (seq & 1) * world * rank_stride;
  bool ok = true;
  for (int64_t e = c * total / G + threadIdx.x; e < e1 && ok; e += CONSUMERS) {
    uint2 v[kMaxTpWorld];
#pragma unroll
    for (int rk = 0; rk < kMaxTpWorld; ++rk)
      if (rk < world) v[rk] = ld_tagged_sys(base + rk * rank_stride + e);
    const uint64_t t0 = globaltimer();
#pragma unroll
    for (int rk = 0; rk < kMaxTpWorld; ++rk) {
      if (rk < world && ok) {
        while (static_cast<int>(v[rk].y) != seq + 1) {
          if (*reinterpret_cast<volatile int*>(status) != 0 || globaltimer() - t0 > kWaitNs) {
            atomicOr(status, kStatusTpTimeout);
            ok = false;
            break;
          }
          __nanosleep(32);
          v[rk] = ld_tagged_sys(base + rk * rank_stride + e);
        }
      }
    }
    if (ok) {
      float sum = 0.f;
#pragma unroll
      for (int rk = 0; rk < kMaxTpWorld; ++rk)
        if (rk < world) sum += __uint_as_float(v[rk].x);
      out[e] = from_f32<T>(sum + to_f32(res[e]));
    }
  }
  return ok;
}

// TP = false: phases gate/up, down (+ residual).  TP = true: gate/up, down
// (partials published to every rank), reduce (+ residual).
template <typename T, int NT, bool TP>
__global__ void __launch_bounds__(kStackThreads, 1) mlp_stack_kernel(const __grid_constant__ StackParams p) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ int s_last, s_abort;
  __shared__ float s_sumsq[GW][MT_MAX];
  __shared__ __align__(8) uint64_t s_mid[2];
  __shared__ __align__(8) uint64_t s_nw_full, s_nw_empty;
  __shared__ int s_mid_last, s_fast, s_decided;
  __shared__ const void* s_hidden;  // this layer's input rows (the gate/up phase's norm reads them)
  __shared__ int s_seq0;            // tensor parallel: the exchange round of this launch's first layer
  // This CTA's step ranges and phase grids, kept in shared memory and read
  // where used, so they hold no registers across the streaming loops.
  __shared__ int64_t s_rng[6];

  constexpr int PPL = TP ? 3 : 2;  // phases per layer
  const GemvArgs& ga = p.ga;
  const GemvArgs& da = p.da;
  const Ring r = carve_ring(smem_raw, ga.stages, ga.boxes, 0, p.x_bytes);
  unsigned char* nw_smem = r.xreg + p.xact_bytes;
  const int nes = ga.norm_dtype == FD_F32 ? 4 : 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = kStackProducers;
  // Each phase is split over min(grid, its steps) CTAs -- the grid of a
  // single launch of that shape -- so the sums match the chain's bit for
  // bit; CTAs past that have an empty range and only take part in barriers.
  const int64_t G = gridDim.x, c = blockIdx.x;
  const int64_t Gg = G < ga.total ? G : ga.total, Gd = G < da.total ? G : da.total;
  const int64_t g0 = c < Gg ? range_start(c, ga.total, Gg) : 0, g1 = c < Gg ? range_start(c + 1, ga.total, Gg) : 0;
  const int64_t d0 = c < Gd ? range_start(c, da.total, Gd) : 0, d1 = c < Gd ? range_start(c + 1, da.total, Gd) : 0;
  const int nphase = PPL * p.layers;
  const int gmid = has_mid_block(g0, g1, ga.ks) ? 1 : 0, dmid = has_mid_block(d0, d1, da.ks) ? 1 : 0;
  // mid-block hand-offs before phase ph: the parity of this phase's MidSync mbarriers
  auto mid_parity = [&](int ph) -> uint32_t {
    const int k = ph % PPL;
    return static_cast<uint32_t>((ph / PPL) * (gmid + dmid) + (k >= 1 ? gmid : 0) + (k >= 2 ? dmid : 0)) & 1u;
  };
  auto sync_for = [&](int ph) {
    return MidSync{&s_mid[0], &s_mid[1], &s_mid_last, &s_fast, &s_decided, mid_parity(ph), ph + 1};
  };
  int* status = ga.status;

  if (threadIdx.x == 0) {
    mbar_init(&s_mid[0], GW);
    mbar_init(&s_mid[1], 1);
    mbar_init(&s_nw_full, 1);
    mbar_init(&s_nw_empty, 1);
    ring_init(r);  // ends with the mbarrier-init fence
    s_abort = 0;
    s_fast = 0;
    s_decided = 0;
    s_rng[0] = g0; s_rng[1] = g1; s_rng[2] = d0; s_rng[3] = d1; s_rng[4] = Gg; s_rng[5] = Gd;
  }
  __syncthreads();

  if (warp >= GW) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kHelperRegs));
    if (warp == GW + P + 1) return;  // the idle warp of the helper warpgroup
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));
  }

  if (warp == GW + P) {
    // announcer: each phase's mid-block publication, and in gate/up phases
    // the watch on the final block's counter
    grid_dep_wait();
    if (lane == 0) {
      // the round number only changes at the very end of this kernel (below)
      const int seq0 = TP ? *reinterpret_cast<volatile int*>(p.tp_buf) : 0;
      for (int ph = 0; ph < nphase; ++ph) {
        const int k = ph % PPL;
        // the split-K counters of this phase are clean once the previous phase is done
        if (ph > 0 && !phase_wait(p.bar, static_cast<int>(G) * ph, status, &s_abort)) break;
        if (k < 2) {
          const GemvArgs& a = k == 0 ? ga : da;
          const MidSync ms = sync_for(ph);
          announce_mid(a, ms, k == 0 ? g0 : d0, k == 0 ? g1 : d1, k == 0 ? Gg : Gd, &s_abort);
          if (k == 0) watch_final(a, ms, g0, g1, Gg, c);
        }
        if (*reinterpret_cast<volatile int*>(&s_abort)) break;
        if (ph == nphase - 1 && phase_wait(p.bar, static_cast<int>(G) * nphase, status, &s_abort)) {
          // every CTA has finished the launch's last phase and has no count left to wait for
          int* depart = p.bar + kDepartOffset;
          if (atomicAdd(depart, 1) == static_cast<int>(G) - 1) {
            if (TP) *reinterpret_cast<volatile int*>(p.tp_buf) = seq0 + p.layers;  // rounds used by this launch
            *reinterpret_cast<volatile int*>(p.bar) = 0;
            *reinterpret_cast<volatile int*>(depart) = 0;
          }
        }
      }
    }
    return;
  }

  if (warp >= GW) {
    // producers: weights only, phase after phase, ring indices continuing
    const int pi = warp - GW;
    if (lane == 0) {
      const uint64_t pol = evict_first_policy();
      const uint32_t nb = static_cast<uint32_t>(ga.k * nes);
      int64_t base = 0;
      for (int l = 0; l < p.layers; ++l) {
        if (pi == 0) {
          // layer l's norm weight, once the consumers are done with layer l-1's
          if (l > 0 && !mbar_wait(&s_nw_empty, static_cast<uint32_t>((l - 1) & 1))) {
            atomicOr(status, kStatusEmptyTimeout);
            s_abort = 1;
            break;
          }
          mbar_expect_tx(&s_nw_full, nb);
          bulk_load(nw_smem, p.norm_w[l], nb, &s_nw_full);
        }
        prefetch_map(&p.gu[l]);
        prefetch_map(&p.dn[l]);
        const auto ready = [] { return true; };
        if (!produce_phase<MODE_GATEUP>(r, &p.gu[l], &p.gu[l], ga, g0, g1, base, pi, P, pol, &s_abort, ready))
          break;
        base += g1 - g0;
        if (!produce_phase<MODE_LINEAR_X>(r, &p.dn[l], &p.dn[l], da, d0, d1, base, pi, P, pol, &s_abort, ready))
          break;
        base += d1 - d0;
      }
      producer_drain(r, static_cast<int64_t>(p.layers) * ((g1 - g0) + (d1 - d0)), pi, P);
    }
    return;
  }

  // consumers
  grid_dep_wait();
  if (TP && threadIdx.x == 0) s_seq0 = *reinterpret_cast<volatile int*>(p.tp_buf);
  const volatile int64_t* rng = s_rng;
  int64_t base = 0;
  for (int l = 0; l < p.layers; ++l) {
    const int ph = PPL * l;
    const int gl = p.first_layer + l;
    // ---- gate/up of layer l
    if (ph > 0 && !consumer_phase_wait(p.bar, static_cast<int>(gridDim.x) * ph, status, &s_abort)) break;
    if (threadIdx.x == 0) s_hidden = gl == 0 ? p.hidden : p.ping[(gl - 1) & 1];
    consumer_sync();
    norm_to_smem<T, 1>(ga, *reinterpret_cast<const void* volatile*>(&s_hidden), r, s_sumsq, nw_smem, &s_nw_full,
                    static_cast<uint32_t>(l & 1));
    if (threadIdx.x == 0) mbar_arrive(&s_nw_empty);
    if (!consume_phase<T, NT, 0, 1, MODE_GATEUP>(ga, r, rng[0], rng[1], base, rng[4], blockIdx.x, &s_last,
                                                 &s_abort, sync_for(ph)))
      break;
    base += rng[1] - rng[0];
    phase_arrive(p.bar);
    // ---- down of layer l: + hidden_l, or (tensor parallel) the partial to every rank
    if (!consumer_phase_wait(p.bar, static_cast<int>(gridDim.x) * (ph + 1), status, &s_abort)) break;
    if (threadIdx.x == 0) {
      sx_ra = gl == 0 ? p.hidden : p.ping[(gl - 1) & 1];
      sx_y = static_cast<char*>(gl == p.total_layers - 1 ? p.out : p.ping[gl & 1]);
      if (TP) sx_seq = s_seq0 + l;
    }
    stage_x<T>(da, r, static_cast<const T*>(p.mid), rng[2], rng[3]);  // ends with a consumer barrier
    if (!consume_phase<T, NT, 0, 1, MODE_LINEAR_X>(da, r, rng[2], rng[3], base, rng[5], blockIdx.x, &s_last,
                                                   &s_abort, sync_for(ph + 1)))
      break;
    base += rng[3] - rng[2];
    phase_arrive(p.bar);
    if (TP) {
      // ---- reduce of layer l: hidden_{l+1} = round(sum of the ranks' partials + hidden_l)
      if (!consumer_phase_wait(p.bar, static_cast<int>(gridDim.x) * (ph + 2), status, &s_abort)) break;
      const T* res = static_cast<const T*>(gl == 0 ? p.hidden : p.ping[(gl - 1) & 1]);
      T* out = static_cast<T*>(gl == p.total_layers - 1 ? p.out : p.ping[gl & 1]);
      if (!tp_reduce_phase<T>(p, s_seq0 + l, res, out, status)) s_abort = 1;
      phase_arrive(p.bar);
      if (*reinterpret_cast<volatile int*>(&s_abort)) break;
    }
  }
}

// ------------------------------------------------------------ host side
struct StackGeometry {
  int stages, boxes;
  int64_t ks_g, ks_d;
  size_t xact, xbytes, smem;
};

// Ring stages for the stack at batch m: as many as fit (at most 8), after
// the X region (the larger of the gate/up normalised batch and a CTA's
// columns of mid) and the norm weight.  FD_STACK_STAGES overrides.
StackGeometry stack_geometry(int m, int64_t h, int64_t i, int nes, int grid) {
  StackGeometry g;
  g.boxes = 2;
  g.ks_g = (h + g.boxes * KC - 1) / (g.boxes * KC);
  g.ks_d = (i + g.boxes * KC - 1) / (g.boxes * KC);
  const int64_t total_d = ((h + BR - 1) / BR) * g.ks_d;
  const int64_t maxlen_d = (total_d + grid - 1) / grid;
  const size_t x_gu = gateup_x_bytes(m, g.ks_g, g.boxes);
  const size_t x_dn = static_cast<size_t>(maxlen_d) * g.boxes * m * 128;
  g.xact = std::max(x_gu, x_dn);
  g.xbytes = g.xact + ((static_cast<size_t>(h) * nes + 15) & ~static_cast<size_t>(15));
  int want = 8;
  if (const char* env = std::getenv("FD_STACK_STAGES")) {
    const int v = std::atoi(env);
    if (v >= 2 && v <= MAX_STAGES) want = v;
  }
  g.stages = want - want % kStackProducers;
  // this kernel's static shared memory (two argument copies) is larger than the single launches'
  constexpr size_t kLimit = kSmemPerCta - 2048;
  while (g.stages >= 2 && ring_smem_bytes(g.xbytes, g.stages, g.boxes) > kLimit) g.stages -= kStackProducers;
  g.smem = g.stages >= 2 ? ring_smem_bytes(g.xbytes, g.stages, g.boxes) : 0;
  if (g.stages < 2) g.stages = 0;
  return g;
}

template <typename T, int NT, bool TP>
cudaError_t launch_stack(const StackParams& p, int grid, size_t smem, cudaStream_t st) {
  auto kern = mlp_stack_kernel<T, NT, TP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kStackThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

}  // namespace

namespace fd_host {

// Whether a stack runs as the persistent kernel.  Measured on B200 (32-layer
// Llama-3-8B stacks in CUDA graphs, same box, same call): on one GPU the
// launch chain is as fast or faster at every batch (M=1 66.4 vs 70.4
// us/layer, M=8 72.3 vs 82.1), and tensor parallel over 2 GPUs too (M=1
// 46.2 vs 55.7 us/layer with the rank reduction inside the kernel): a phase
// boundary inside the kernel costs what a kernel boundary costs -- the
// slowest SM's tail, the barrier and the activation round trip -- and the
// chain's launches each get a ring sized for their own phase.  So the
// persistent kernel is opt-in (FD_STACK_PERSISTENT=1), and needs at least 4
// ring stages.
bool persistent_wanted(bool /*tp*/, const StackGeometry& geo) {
  if (geo.stages < 4) return false;
  const char* env = std::getenv("FD_STACK_PERSISTENT");
  return env && env[0] == '1';
}

// The persistent stack for `layers` layers (weights as arrays of device
// pointers).  Returns FD_ERR_UNSUPPORTED when this shape is not served by the
// persistent kernel (the caller then runs the launch chain).  With tp_world
// > 0 the layers are tensor-parallel shards (i is this rank's share of the
// intermediate width) and the partial sums travel through `exchange`.
int mlp_stack_persistent(const void* hidden, int32_t layers, const void* const* norm_w, int32_t norm_dtype,
                         const void* const* w_gate_up, int64_t s_gu, const void* const* w_down, int64_t s_down,
                         void* out, int32_t dtype, int32_t m, int64_t h, int64_t i, float eps, int32_t kind,
                         const fd_stream::Workspace& ws, void* mid, void* ping0, void* ping1, cudaStream_t st,
                         int32_t tp_rank, int32_t tp_world, void* const* exchange, int32_t tp_mmax) {
  if (kind != FD_KIND_DOT || m < 1 || m > MT_MAX || layers < 1) return FD_ERR_UNSUPPORTED;
  const int nes = norm_dtype == FD_F32 ? 4 : 2;
  const int grid = sm_count();
  const StackGeometry geo = stack_geometry(m, h, i, nes, grid);
  if (!persistent_wanted(tp_world > 0, geo)) return FD_ERR_UNSUPPORTED;

  StackParams p;
  std::memset(&p, 0, sizeof(p));
  GemvArgs& ga = p.ga;
  ga.y = static_cast<char*>(mid); ga.sym = i; ga.syn = 1;
  ga.m = m; ga.n = 2 * i; ga.k = h;
  ga.boxes = geo.boxes; ga.stages = geo.stages; ga.ks = geo.ks_g;
  ga.nblocks = (i + BR / 2 - 1) / (BR / 2);
  ga.total = ga.nblocks * ga.ks;
  ga.slots = ws.slots; ga.counters = ws.counters; ga.status = ws.status;
  ga.inner = i;
  ga.hidden_stride = h;
  ga.norm_dtype = norm_dtype; ga.eps = eps;
  GemvArgs& da = p.da;
  da.ra_dtype = dtype; da.srm = h; da.srn = 1;
  da.sym = h; da.syn = 1;
  da.m = m; da.n = h; da.k = i;
  da.boxes = geo.boxes; da.stages = geo.stages; da.ks = geo.ks_d;
  da.nblocks = (h + BR - 1) / BR;
  da.total = da.nblocks * da.ks;
  da.slots = ws.slots; da.counters = ws.counters; da.status = ws.status;
  if (ga.nblocks > kMaxCounters || da.nblocks > kMaxCounters) return FD_ERR_UNSUPPORTED;
  const bool tp = tp_world > 0;
  if (tp) {
    const TpLayout lay = tp_layout(tp_world, tp_mmax, h);
    for (int k = 0; k < tp_world; ++k) da.tp_peer[k] = static_cast<char*>(exchange[k]);
    da.tp_rank = tp_rank; da.tp_world = tp_world; da.tp_mmax = tp_mmax;
    da.tp_data_off = lay.data_off;
    p.tp_buf = static_cast<char*>(exchange[tp_rank]);
  }
  p.hidden = hidden;
  p.out = out;
  p.ping[0] = static_cast<char*>(ping0);
  p.ping[1] = static_cast<char*>(ping1);
  p.mid = mid;
  p.bar = reinterpret_cast<int*>(reinterpret_cast<char*>(ws.status) + kBarOffset);
  p.total_layers = layers;
  p.xact_bytes = static_cast<int>(geo.xact);
  p.x_bytes = static_cast<int>(geo.xbytes);

  for (int l0 = 0; l0 < layers; l0 += kStackMaxLayers) {
    const int n = std::min(kStackMaxLayers, layers - l0);
    p.first_layer = l0;
    p.layers = n;
    for (int l = 0; l < n; ++l) {
      if (!make_gate_up_map(&p.gu[l], w_gate_up[l0 + l], h, i, s_gu) ||
          !make_map_2d(&p.dn[l], w_down[l0 + l], h, i, s_down, BR))
        return FD_ERR_LAUNCH;
      p.norm_w[l] = norm_w[l0 + l];
    }
    cudaError_t e;
    const bool wide = m > 8;
    if (dtype == FD_BF16) {
      if (tp) e = wide ? launch_stack<__nv_bfloat16, 2, true>(p, grid, geo.smem, st)
                       : launch_stack<__nv_bfloat16, 1, true>(p, grid, geo.smem, st);
      else e = wide ? launch_stack<__nv_bfloat16, 2, false>(p, grid, geo.smem, st)
                    : launch_stack<__nv_bfloat16, 1, false>(p, grid, geo.smem, st);
    } else {
      if (tp) e = wide ? launch_stack<__half, 2, true>(p, grid, geo.smem, st)
                       : launch_stack<__half, 1, true>(p, grid, geo.smem, st);
      else e = wide ? launch_stack<__half, 2, false>(p, grid, geo.smem, st)
                    : launch_stack<__half, 1, false>(p, grid, geo.smem, st);
    }
    if (e != cudaSuccess) return FD_ERR_LAUNCH;
  }
  return FD_OK;
}

int mlp_stack_launches(int32_t layers, int32_t norm_dtype, int32_t m, int64_t h, int64_t i, int32_t kind) {
  if (layers <= 0 || m <= 0 || h <= 0) return 0;
  const bool persistent =
      kind == FD_KIND_DOT && m <= MT_MAX &&
      persistent_wanted(false, stack_geometry(m, h, i, norm_dtype == FD_F32 ? 4 : 2, sm_count()));
  return persistent ? (layers + kStackMaxLayers - 1) / kStackMaxLayers
                    : layers * mlp_layer_launches(m, h, i, norm_dtype, kind, false);
}

}  // namespace fd_host

extern "C" int fd_post_attn_mlp_tp_stack_launches(int32_t layers, int32_t norm_dtype, int32_t m, int64_t h,
                                                  int64_t i, int32_t kind) {
  if (layers <= 0 || m <= 0 || h <= 0) return 0;
  const bool persistent =
      kind == FD_KIND_DOT && m <= MT_MAX &&
      fd_host::persistent_wanted(true, stack_geometry(m, h, i, norm_dtype == FD_F32 ? 4 : 2, fd_host::sm_count()));
  if (persistent) return (layers + kStackMaxLayers - 1) / kStackMaxLayers;
  return layers * fd_host::mlp_layer_launches(m, h, i, norm_dtype, kind, true);
}

extern "C" int fd_post_attn_mlp_layer_launches(int32_t m, int64_t h, int64_t i, int32_t norm_dtype, int32_t kind,
                                               int32_t tensor_parallel) {
  if (m <= 0 || h <= 0) return 0;
  return fd_host::mlp_layer_launches(m, h, i, norm_dtype, kind, tensor_parallel != 0);
}

extern "C" int fd_post_attn_mlp_stack_launches(int32_t layers, int32_t norm_dtype, int32_t m, int64_t h, int64_t i,
                                               int32_t kind) {
  return fd_host::mlp_stack_launches(layers, norm_dtype, m, h, i, kind);
}
