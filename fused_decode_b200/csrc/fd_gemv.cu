// Small-batch GEMV family (M = 1..16) and the fused post-attention MLP.
//
// Design (sm_100a, HBM-bound):
//  * Stream-K over the weight.  The weight is cut into blocks of BR rows; each
//    block is a run of KS "steps" of 32 columns.  The grid (a multiple of the
//    SM count) splits the flat step range [0, nblocks*KS) into equal contiguous
//    pieces, so every CTA streams the same number of weight bytes whatever N
//    and K are (the reference grid is cdiv(N, 64) CTAs with no split-K,
//    kernels.py:775, which leaves most SMs idle at N=4096).
//  * Each warp owns 16 rows of the block.  Per step a lane issues two 16-byte
//    loads (rows g and g+8, columns 8q..8q+7 of the step, g = lane/4,
//    q = lane%4) and keeps D steps in flight in a register ring.
//  * "dot" kind: the 16 x 32 tile feeds two mma.sync m16n8k16 (swap-AB: the
//    weight is the A operand, the batch is N=8 or 16).  The 32 physical columns
//    a lane holds are assigned to logical MMA k-indices by a fixed permutation
//    that is applied identically to A and B, so the sum is unchanged and the
//    loads stay 16 bytes wide.
//  * "simt" kind: the same loads, fp32 FMAs against all M rows of x, then a
//    4-lane shuffle reduction.
//  * Split-K partials go to per-CTA slots in a workspace; the last CTA to
//    finish a block (an atomic counter) sums the slots in CTA order --
//    deterministic, no spin-wait -- applies the epilogue and re-zeroes the
//    counter so the workspace is ready for the next launch / graph replay.
//  * The fused MLP's gate/up kernel computes RMSNorm of the (tiny) hidden
//    batch into shared memory in its prologue, pairs 64 gate rows with the
//    matching 64 up rows in each block, and applies SwiGLU in the epilogue;
//    the down kernel adds the residual in its epilogue.  Both launch with
//    programmatic dependent launch: the weight prefetch of the next kernel
//    is issued before griddepcontrol.wait.
#include "fd_common.cuh"

#include <algorithm>

using namespace fd;

namespace {

constexpr int GW = 8;           // warps per CTA
constexpr int BR = GW * 16;     // weight rows per block
constexpr int KSTEP = 32;       // columns per step
constexpr int MT_MAX = 16;      // max batch rows
constexpr int XPAD = 64;        // bytes of padding per shared x row: pitch = 64 mod 128 B,
                                // so the 8 lanes of a 16-byte load phase hit distinct banks

enum Mode { MODE_LINEAR = 0, MODE_GATEUP = 1 };

struct GemvArgs {
  // operands (all strides in elements; k-stride of x and w is 1)
  const char* x;
  int64_t sxm;
  const char* w;
  int64_t swn;
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
  float* slots;     // [grid][2][BR * MT_MAX]
  int* counters;    // [nblocks]
  // gate/up mode
  int64_t inner;            // I: up rows start at row I of w
  const void* hidden;       // [m, k] contiguous rows (row stride hidden_stride)
  int64_t hidden_stride;
  const void* norm_w;
  int32_t norm_dtype;
  float eps;
  int32_t xs_pitch;         // shared x row pitch in elements
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

// Weight stream: read once, do not keep in L1, evict early from L2.
FD_DEV uint4 ld_weight16(const void* p, uint64_t policy) {
  uint4 v;
  asm volatile(
      "ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "l"(policy));
  return v;
}
FD_DEV uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
FD_DEV uint4 lds16(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}
FD_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
FD_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------ stream-K split
FD_DEV int64_t range_start(int64_t c, int64_t total, int64_t G) { return c * total / G; }
// The CTA whose range holds step t.
FD_DEV int64_t cta_of(int64_t t, int64_t total, int64_t G) { return ((t + 1) * G - 1) / total; }

FD_DEV float silu_mul(float g, float u) {
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
};

// ------------------------------------------------------------ epilogues
template <typename T, int NT, int MODE>
struct Epilogue;

// Plain linear: y = round(acc + bias + row_add).
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
    __syncthreads();
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
    __syncthreads();
  }
};

// ------------------------------------------------------------ the kernel
// KIND 0 = dot (mma.sync), 1 = simt.  MP = padded batch for simt (1..16).
// XS = x lives in shared memory (gate/up mode with the norm fused).
template <typename T, int NT, int KIND, int MP, int MODE, bool XS, int D>
__global__ void __launch_bounds__(GW * 32, 2) gemv_streamk_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t G = gridDim.x, c = blockIdx.x;
  const int64_t s0 = range_start(c, a.total, G);
  const int64_t s1 = range_start(c + 1, a.total, G);
  const uint64_t pol = evict_first_policy();

  T* xs = reinterpret_cast<T*>(smem);  // [m][xs_pitch] when XS
  float* xchg = reinterpret_cast<float*>(smem + (XS ? static_cast<size_t>(a.m) * a.xs_pitch * sizeof(T) : 0));

  // Weight row of this lane for block `blk` and half `hh` (row g or g+8).
  auto wrow = [&](int64_t blk, int hh, bool& ok) -> const T* {
    int64_t r;
    if (MODE == MODE_GATEUP) {
      const int w4 = warp & (GW / 2 - 1);
      const int64_t j = blk * (BR / 2) + 16 * w4 + g + 8 * hh;
      ok = j < a.inner;
      r = (warp >= GW / 2) ? a.inner + j : j;
    } else {
      r = blk * BR + 16 * warp + g + 8 * hh;
      ok = r < a.n;
    }
    return reinterpret_cast<const T*>(a.w) + (ok ? r : 0) * a.swn;
  };

  // -------- register ring
  uint4 ra_[D], rb_[D], rx_[D][NT];
  // load cursor
  int64_t lt = s0, lb = s0 / a.ks, lk = s0 - (s0 / a.ks) * a.ks;
  bool ok0, ok1;
  const T* wr0 = wrow(lb, 0, ok0);
  const T* wr1 = wrow(lb, 1, ok1);

  auto load_w = [&](int i) {
    const int64_t col = lk * KSTEP + 8 * q;
    const bool kin = col < a.k;
    ra_[i] = (ok0 && kin) ? ld_weight16(wr0 + col, pol) : make_uint4(0, 0, 0, 0);
    rb_[i] = (ok1 && kin) ? ld_weight16(wr1 + col, pol) : make_uint4(0, 0, 0, 0);
  };
  auto load_x = [&](int i, int64_t kk) {
    if (KIND == 0) {
      const int64_t col = kk * KSTEP + 8 * q;
      const bool kin = col < a.k;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int mrow = g + 8 * t;
        if (kin && mrow < a.m) {
          if (XS)
            rx_[i][t] = lds16(xs + mrow * a.xs_pitch + col);
          else
            rx_[i][t] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.x) + mrow * a.sxm + col));
        } else {
          rx_[i][t] = make_uint4(0, 0, 0, 0);
        }
      }
    }
  };
  auto advance_load = [&]() {
    ++lt;
    if (++lk == a.ks) {
      lk = 0;
      ++lb;
      wr0 = wrow(lb, 0, ok0);
      wr1 = wrow(lb, 1, ok1);
    }
  };

  // Prologue part 1: weight prefetch (independent of the previous kernel).
  int64_t kk_of_stage[D];
#pragma unroll
  for (int i = 0; i < D; ++i) {
    kk_of_stage[i] = lk;
    if (lt < s1) {
      load_w(i);
      advance_load();
    }
  }

  // Everything below may read the previous kernel's outputs.
  grid_dep_wait();

  if (XS) {
    // RMSNorm of the m hidden rows into shared memory, rounded to T
    // (reference.py:389 rounds `normed` to the activation dtype).
    const int nvec = static_cast<int>(a.k / 8);
    for (int mrow = warp; mrow < a.m; mrow += GW) {
      const T* hr = reinterpret_cast<const T*>(a.hidden) + mrow * a.hidden_stride;
      float ss = 0.f;
      for (int v = lane; v < nvec; v += 32) {
        float f[8];
        unpack8<T>(__ldg(reinterpret_cast<const uint4*>(hr) + v), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
      }
      ss = warp_sum(ss);
      const float inv = 1.0f / sqrtf(ss / static_cast<float>(a.k) + a.eps);
      const int wes = a.norm_dtype == FD_F32 ? 4 : 2;
      for (int v = lane; v < nvec; v += 32) {
        float f[8], wv[8], o[8];
        unpack8<T>(__ldg(reinterpret_cast<const uint4*>(hr) + v), f);
        load8_as_f32(static_cast<const char*>(a.norm_w) + static_cast<int64_t>(v) * 8 * wes, a.norm_dtype, wv);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = f[e] * inv * wv[e];
        *reinterpret_cast<uint4*>(xs + mrow * a.xs_pitch + 8 * v) = pack8<T>(o);
      }
    }
    __syncthreads();
  }
  grid_dep_launch();

#pragma unroll
  for (int i = 0; i < D; ++i) load_x(i, kk_of_stage[i]);

  // -------- main loop
  int64_t ct = s0, cb = s0 / a.ks, ck = s0 - (s0 / a.ks) * a.ks;
  Acc<NT> acc;
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc.v[t][e] = 0.f;
  float sacc[2][MP];  // simt accumulators
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int mm = 0; mm < MP; ++mm) sacc[r][mm] = 0.f;

  while (ct < s1) {
#pragma unroll
    for (int i = 0; i < D; ++i) {
      if (ct < s1) {
        // ---- compute stage i (step ct, column block ck)
        if (KIND == 0) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            mma16816<T>(acc.v[t], ra_[i].x, rb_[i].x, ra_[i].y, rb_[i].y, rx_[i][t].x, rx_[i][t].y);
            mma16816<T>(acc.v[t], ra_[i].z, rb_[i].z, ra_[i].w, rb_[i].w, rx_[i][t].z, rx_[i][t].w);
          }
        } else {
          const int64_t col = ck * KSTEP + 8 * q;
          if (col < a.k) {
            float wa[8], wb[8];
            unpack8<T>(ra_[i], wa);
            unpack8<T>(rb_[i], wb);
#pragma unroll
            for (int mm = 0; mm < MP; ++mm) {
              if (mm < a.m) {
                uint4 xv;
                if (XS)
                  xv = lds16(xs + mm * a.xs_pitch + col);
                else
                  xv = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.x) + mm * a.sxm + col));
                float xf[8];
                unpack8<T>(xv, xf);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  sacc[0][mm] = fmaf(wa[e], xf[e], sacc[0][mm]);
                  sacc[1][mm] = fmaf(wb[e], xf[e], sacc[1][mm]);
                }
              }
            }
          }
        }
        // ---- refill stage i with the step D ahead
        if (lt < s1) {
          const int64_t kk = lk;
          load_w(i);
          load_x(i, kk);
          advance_load();
        }
        ++ct;
        ++ck;
        // ---- block finished (or range ends): flush
        if (ck == a.ks || ct == s1) {
          if (KIND == 1) {
            // reduce the four q-lanes and move to the C-fragment ownership
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
          const int64_t blk = cb;
          const bool covered = (s0 <= blk * a.ks) && (s1 >= (blk + 1) * a.ks);
          if (covered) {
            Epilogue<T, NT, MODE>::run(a, blk, acc, xchg);
          } else {
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
            __syncthreads();
            const int64_t cf = cta_of(blk * a.ks, a.total, G);
            const int64_t cl = cta_of((blk + 1) * a.ks - 1, a.total, G);
            if (threadIdx.x == 0) {
              const int old = atomicAdd(a.counters + blk, 1);
              s_last = (old == static_cast<int>(cl - cf));
            }
            __syncthreads();
            if (s_last) {
              __threadfence();
              Acc<NT> sum;
#pragma unroll
              for (int t = 0; t < NT; ++t)
#pragma unroll
                for (int e = 0; e < 4; ++e) sum.v[t][e] = 0.f;
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
#pragma unroll
          for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc.v[t][e] = 0.f;
#pragma unroll
          for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int mm = 0; mm < MP; ++mm) sacc[r][mm] = 0.f;
          ck = 0;
          ++cb;
        }
      }
    }
  }
}

// ------------------------------------------------------------ generic GEMV
// Any strides, any K: one warp per output row.  Used for layouts the
// streaming kernel cannot address (transposed weights, K % 8 != 0, ...).
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
    float bias = a.bias ? load_as_f32(a.bias, a.bias_dtype, row * a.sbias) : 0.f;
#pragma unroll
    for (int mm = 0; mm < MT_MAX; ++mm) {
      if (mm < a.m) {
        float v = acc[mm];
        if (a.bias) v += bias;
        if (a.ra) v += load_as_f32(a.ra, a.ra_dtype, mm * a.srm + row * a.srn);
        static_cast<T*>(a.y)[mm * a.sym + row * a.syn] = from_f32<T>(v);
      }
    }
  }
}

// ------------------------------------------------------------ host side
constexpr int kCtasPerSm = 2;
constexpr int kStages = 4;

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

int64_t max_grid() { return static_cast<int64_t>(fd_host::sm_count()) * kCtasPerSm; }

// Workspace: [counters (nblocks ints)] [slots: grid x 2 x BR x MT_MAX floats]
size_t streamk_ws_bytes(int64_t nblocks) {
  return align256(static_cast<size_t>(nblocks) * sizeof(int)) +
         align256(static_cast<size_t>(max_grid()) * 2 * BR * MT_MAX * sizeof(float));
}

template <typename Kern>
cudaError_t launch_pdl(Kern kern, int64_t total, size_t smem, cudaStream_t st, const GemvArgs& a) {
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  // One wave: as many CTAs as fit at once (at most kCtasPerSm per SM), never
  // more than there are steps, so every CTA owns a non-empty step range.
  int occ = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, GW * 32, smem);
  if (e != cudaSuccess) return e;
  occ = std::max(1, std::min(occ, kCtasPerSm));
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(static_cast<int64_t>(fd_host::sm_count()) * occ, total));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(GW * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <typename T, int MODE, bool XS>
cudaError_t launch_streamk(const GemvArgs& a, int kind, size_t smem, cudaStream_t st) {
  const int64_t grid = a.total;
  if (kind == FD_KIND_DOT) {
    if (a.m <= 8) return launch_pdl(gemv_streamk_kernel<T, 1, 0, 1, MODE, XS, kStages>, grid, smem, st, a);
    return launch_pdl(gemv_streamk_kernel<T, 2, 0, 1, MODE, XS, kStages>, grid, smem, st, a);
  }
  if (a.m <= 1) return launch_pdl(gemv_streamk_kernel<T, 1, 1, 1, MODE, XS, kStages>, grid, smem, st, a);
  if (a.m <= 2) return launch_pdl(gemv_streamk_kernel<T, 1, 1, 2, MODE, XS, kStages>, grid, smem, st, a);
  if (a.m <= 4) return launch_pdl(gemv_streamk_kernel<T, 1, 1, 4, MODE, XS, kStages>, grid, smem, st, a);
  if (a.m <= 8) return launch_pdl(gemv_streamk_kernel<T, 1, 1, 8, MODE, XS, kStages>, grid, smem, st, a);
  return launch_pdl(gemv_streamk_kernel<T, 2, 1, 16, MODE, XS, kStages>, grid, smem, st, a);
}

int from_cuda(cudaError_t e) { return e == cudaSuccess ? FD_OK : FD_ERR_LAUNCH; }

int check_mlp_args(const void* hidden, const void* norm_w, int32_t norm_dtype, const void* w_gate_up,
                   int64_t s_gu, int32_t dtype, int32_t m, int64_t h, int64_t i, int32_t kind) {
  using namespace fd_host;
  if (m < 0 || h < 0 || i < 0) return FD_ERR_ARG;
  if (m > MT_MAX) return FD_ERR_UNSUPPORTED;
  if (!hidden || !norm_w || !w_gate_up) return FD_ERR_ARG;
  if (!half_dtype(dtype) || !valid_dtype(norm_dtype)) return FD_ERR_ARG;
  if (kind != FD_KIND_DOT && kind != FD_KIND_SIMT) return FD_ERR_ARG;
  if (h % 8 || i % 8 || i == 0 || s_gu % 8) return FD_ERR_UNSUPPORTED;
  if (!aligned16(hidden) || !aligned16(norm_w) || !aligned16(w_gate_up)) return FD_ERR_UNSUPPORTED;
  // RMSNorm'd batch lives in shared memory next to the gate/up exchange tile.
  if (static_cast<size_t>(m) * (h + XPAD / 2) * 2 + static_cast<size_t>(BR / 2) * MT_MAX * sizeof(float) >
      200 * 1024)
    return FD_ERR_UNSUPPORTED;
  return FD_OK;
}

// Kernel 1 of the MLP: RMSNorm (prologue) -> gate/up GEMV -> SwiGLU -> mid.
cudaError_t launch_gate_up(const void* hidden, const void* norm_w, int32_t norm_dtype,
                           const void* w_gate_up, int64_t s_gu, void* mid, int64_t s_mid,
                           int32_t dtype, int32_t m, int64_t h, int64_t i, float eps, int32_t kind,
                           int* counters, float* slots, cudaStream_t st) {
  GemvArgs a = {};
  a.w = static_cast<const char*>(w_gate_up); a.swn = s_gu;
  a.y = static_cast<char*>(mid); a.sym = s_mid; a.syn = 1;
  a.m = m; a.n = 2 * i; a.k = h;
  a.ks = (h + KSTEP - 1) / KSTEP;
  a.nblocks = (i + BR / 2 - 1) / (BR / 2);
  a.total = a.nblocks * a.ks;
  a.counters = counters; a.slots = slots;
  a.inner = i;
  a.hidden = hidden; a.hidden_stride = h;
  a.norm_w = norm_w; a.norm_dtype = norm_dtype; a.eps = eps;
  a.xs_pitch = static_cast<int32_t>(h + XPAD / 2);  // elements (2-byte types)
  const size_t smem = static_cast<size_t>(m) * a.xs_pitch * 2 + static_cast<size_t>(BR / 2) * MT_MAX * sizeof(float);
  return dtype == FD_BF16 ? launch_streamk<__nv_bfloat16, MODE_GATEUP, true>(a, kind, smem, st)
                          : launch_streamk<__half, MODE_GATEUP, true>(a, kind, smem, st);
}

}  // namespace

extern "C" {

size_t fd_linear_workspace_bytes(int32_t m, int64_t n, int64_t k) {
  (void)m;
  (void)k;
  const int64_t nblocks = (n + BR - 1) / BR;
  return streamk_ws_bytes(std::max<int64_t>(nblocks, 1));
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
  const bool bf = dtype == FD_BF16;

  const bool fast = k > 0 && swk == 1 && sxk == 1 && k % 8 == 0 && aligned16(x) && aligned16(w) &&
                    swn % 8 == 0 && (m == 1 || sxm % 8 == 0);
  if (fast) {
    GemvArgs a = {};
    a.x = static_cast<const char*>(x); a.sxm = sxm;
    a.w = static_cast<const char*>(w); a.swn = swn;
    a.bias = bias; a.bias_dtype = bias_dtype; a.sbias = sbias;
    a.ra = row_add; a.ra_dtype = ra_dtype; a.srm = srm; a.srn = srn;
    a.y = static_cast<char*>(y); a.sym = sym; a.syn = syn;
    a.m = m; a.n = n; a.k = k;
    a.ks = (k + KSTEP - 1) / KSTEP;
    a.nblocks = (n + BR - 1) / BR;
    a.total = a.nblocks * a.ks;
    const size_t need = streamk_ws_bytes(a.nblocks);
    if (!workspace || workspace_bytes < need) return FD_ERR_WORKSPACE;
    a.counters = static_cast<int*>(workspace);
    a.slots = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                       align256(static_cast<size_t>(a.nblocks) * sizeof(int)));
    const size_t smem = 0;
    cudaError_t e = bf ? launch_streamk<__nv_bfloat16, MODE_LINEAR, false>(a, kind, smem, st)
                       : launch_streamk<__half, MODE_LINEAR, false>(a, kind, smem, st);
    return from_cuda(e);
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
  if (bf) gemv_generic_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(a);
  else gemv_generic_kernel<__half><<<blocks, 256, 0, st>>>(a);
  return from_cuda(cudaGetLastError());
}

// Fused post-attention MLP.  Workspace layout:
//   [counters: max(nblocks_gu, nblocks_down) ints][slots][mid: m x i of T]
size_t fd_post_attn_mlp_workspace_bytes(int32_t m, int64_t h, int64_t i) {
  const int64_t nb_gu = (i + BR / 2 - 1) / (BR / 2);
  const int64_t nb_dn = (h + BR - 1) / BR;
  const int64_t nb = std::max<int64_t>(1, std::max(nb_gu, nb_dn));
  return streamk_ws_bytes(nb) + align256(static_cast<size_t>(std::max(m, 1)) * i * 2);
}


int fd_mlp_gate_up_out(const void* hidden, const void* norm_w, int32_t norm_dtype, const void* w_gate_up,
                       int64_t s_gu, void* mid, int32_t dtype, int32_t m, int64_t h, int64_t i, float eps,
                       int32_t kind, void* workspace, size_t workspace_bytes, void* stream) {
  const int chk = check_mlp_args(hidden, norm_w, norm_dtype, w_gate_up, s_gu, dtype, m, h, i, kind);
  if (chk != FD_OK) return chk;
  if (m == 0 || h == 0) return FD_OK;
  if (!mid) return FD_ERR_ARG;
  const int64_t nb = (i + BR / 2 - 1) / (BR / 2);
  if (!workspace || workspace_bytes < streamk_ws_bytes(nb)) return FD_ERR_WORKSPACE;
  int* counters = static_cast<int*>(workspace);
  float* slots = reinterpret_cast<float*>(static_cast<char*>(workspace) + align256(static_cast<size_t>(nb) * sizeof(int)));
  return from_cuda(launch_gate_up(hidden, norm_w, norm_dtype, w_gate_up, s_gu, mid, i, dtype, m, h, i, eps,
                                  kind, counters, slots, static_cast<cudaStream_t>(stream)));
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
  if (s_down % 8 || !aligned16(w_down) || !aligned16(out)) return FD_ERR_UNSUPPORTED;
  const size_t need = fd_post_attn_mlp_workspace_bytes(m, h, i);
  if (!workspace || workspace_bytes < need) return FD_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  const int64_t nb_gu = (i + BR / 2 - 1) / (BR / 2);
  const int64_t nb_dn = (h + BR - 1) / BR;
  const int64_t nb = std::max(nb_gu, nb_dn);
  char* ws = static_cast<char*>(workspace);
  int* counters = reinterpret_cast<int*>(ws);
  float* slots = reinterpret_cast<float*>(ws + align256(static_cast<size_t>(nb) * sizeof(int)));
  char* mid = ws + streamk_ws_bytes(nb);

  cudaError_t e = launch_gate_up(hidden, norm_w, norm_dtype, w_gate_up, s_gu, mid, i, dtype, m, h, i, eps,
                                 kind, counters, slots, st);
  if (e != cudaSuccess) return FD_ERR_LAUNCH;

  // Kernel 2: down GEMV (+ residual) -> out [m, h].
  GemvArgs b = {};
  b.x = mid; b.sxm = i;
  b.w = static_cast<const char*>(w_down); b.swn = s_down;
  b.ra = add_residual ? hidden : nullptr; b.ra_dtype = dtype; b.srm = h; b.srn = 1;
  b.y = static_cast<char*>(out); b.sym = h; b.syn = 1;
  b.y_f32 = out_dtype == FD_F32;
  b.m = m; b.n = h; b.k = i;
  b.ks = (i + KSTEP - 1) / KSTEP;
  b.nblocks = nb_dn;
  b.total = b.nblocks * b.ks;
  b.counters = counters; b.slots = slots;
  e = dtype == FD_BF16 ? launch_streamk<__nv_bfloat16, MODE_LINEAR, false>(b, kind, 0, st)
                       : launch_streamk<__half, MODE_LINEAR, false>(b, kind, 0, st);
  return from_cuda(e);
}

}  // extern "C"
