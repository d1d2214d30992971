// Row-wise and elementwise decode kernels for sm_100a:
//   RMSNorm / fused add+RMSNorm, SwiGLU, rotate-half RoPE, and the copy / triad
//   roof kernels.  All are HBM-streaming kernels: 16-byte vector loads and
//   stores, fp32 math, one rounding to the activation dtype per output, and a
//   scalar fallback for any layout the vector path cannot address.
#include "fd_common.cuh"

#include <algorithm>
#include <mutex>
#include <unordered_map>

using namespace fd;

namespace {

// Plain (coherent) 16-byte load without L1 allocation.  Used where an output
// may alias the input (in-place residual), so the non-coherent path is avoided.
FD_DEV uint4 ld_plain16(const void* p) {
  uint4 v;
  asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

struct RowsArg {
  char* ptr;
  int64_t sa, sb, sc, col;
};

RowsArg rows_arg(const fd_rows* r) {
  RowsArg a;
  a.ptr = static_cast<char*>(r ? r->ptr : nullptr);
  a.sa = r ? r->sa : 0;
  a.sb = r ? r->sb : 0;
  a.sc = r ? r->sc : 0;
  a.col = r ? r->col : 0;
  return a;
}

template <typename T>
FD_DEV T* row_ptr(const RowsArg& g, int64_t row, int64_t B, int64_t C) {
  return reinterpret_cast<T*>(g.ptr) + row_base(row, B, C, g.sa, g.sb, g.sc);
}

// ============================================================== RMSNorm
// Vector path: each row is handled by a group of `wpr` warps; every thread
// keeps VPT 8-element vectors of the row in registers, so x and residual are
// read from HBM exactly once (reference two-pass kernels re-read the row,
// kernels.py:299-340).
struct RmsArgs {
  RowsArg x, r, y, ro;
  int64_t B, C, rows;
  int32_t flat;  // the grid has one leading dimension
  const void* w;
  int32_t w_dtype;
  int32_t wpr;   // warps per row
  int32_t rpc;   // rows per CTA
  int32_t nv;    // vectors (8 elements) per row
  int32_t n;
  float eps;
};

// Element offset of row `row` in a row grid.  FLAT: a 2-D grid (one leading
// dimension).  Otherwise the (ia, ib, ic) split in 32-bit arithmetic (the host
// sends grids of 2^32 rows or more to the generic kernel).
struct RowIdx {
  uint32_t ia, ib, ic;
};
template <bool FLAT>
FD_DEV RowIdx split_row(int64_t row, int64_t B, int64_t C) {
  if (FLAT) return {0u, 0u, static_cast<uint32_t>(row)};
  const uint32_t r = static_cast<uint32_t>(row), c = static_cast<uint32_t>(C), b = static_cast<uint32_t>(B);
  const uint32_t t = r / c;
  return {t / b, t % b, r % c};
}
FD_DEV int64_t offset_of(const RowsArg& g, const RowIdx& i) {
  return i.ia * g.sa + i.ib * g.sb + static_cast<int64_t>(i.ic) * g.sc;
}

template <typename T, int VPT, bool HAS_RES, bool STORE_RES, bool FLAT>
__global__ void __launch_bounds__(512) rms_vec_kernel(RmsArgs a) {
  __shared__ float red[32];
  const int group_threads = 32 * a.wpr;
  const int group = threadIdx.x / group_threads;
  const int t = threadIdx.x - group * group_threads;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * a.rpc + group;
  const bool live = row < a.rows;
  const RowIdx ri = split_row<FLAT>(live ? row : 0, a.B, a.C);
  grid_dep_wait();
  grid_dep_launch();

  float s[VPT][8];
  float sumsq = 0.f;
  if (live) {
    const T* xr = reinterpret_cast<const T*>(a.x.ptr) + offset_of(a.x, ri);
    const T* rr = HAS_RES ? reinterpret_cast<const T*>(a.r.ptr) + offset_of(a.r, ri) : nullptr;
    uint4 xv[VPT], rv[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int j = t + i * group_threads;
      if (j < a.nv) {
        xv[i] = ld_plain16(xr + 8 * j);
        if (HAS_RES) rv[i] = ld_plain16(rr + 8 * j);
      }
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int j = t + i * group_threads;
      if (j < a.nv) {
        unpack8<T>(xv[i], s[i]);
        if (HAS_RES) {
          float rf[8];
          unpack8<T>(rv[i], rf);
#pragma unroll
          for (int e = 0; e < 8; ++e) s[i][e] += rf[e];
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) sumsq += s[i][e] * s[i][e];
      }
    }
    if (STORE_RES) {
      T* ror = reinterpret_cast<T*>(a.ro.ptr) + offset_of(a.ro, ri);
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int j = t + i * group_threads;
        if (j < a.nv) st_stream16(ror + 8 * j, pack8<T>(s[i]));
      }
    }
  }
  sumsq = warp_sum(sumsq);
  if (a.wpr > 1) {
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = sumsq;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < a.wpr; ++w) tot += red[group * a.wpr + w];
    sumsq = tot;
  }
  if (!live) return;
  const float inv = rsqrtf(sumsq / static_cast<float>(a.n) + a.eps);  // rsqrt, as the reference
  T* yr = reinterpret_cast<T*>(a.y.ptr) + offset_of(a.y, ri);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int j = t + i * group_threads;
    if (j < a.nv) {
      float w[8];
      load8_as_f32(static_cast<const char*>(a.w) + static_cast<int64_t>(8 * j) * (a.w_dtype == FD_F32 ? 4 : 2),
                   a.w_dtype, w);
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = s[i][e] * inv * w[e];
      st_stream16(yr + 8 * j, pack8<T>(o));
    }
  }
}

// Generic path: any strides, any n.  One CTA per row, two passes over the row
// (the second pass re-reads x/residual from L2).
struct RmsGenArgs {
  RowsArg x, r, y, ro;
  int64_t B, C, rows;
  const void* w;
  int32_t w_dtype;
  int64_t w_stride;
  int64_t n;
  float eps;
  int has_res, store_res;
};

template <typename T>
__global__ void __launch_bounds__(256) rms_generic_kernel(RmsGenArgs a) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  grid_dep_wait();
  grid_dep_launch();
  const T* xr = row_ptr<T>(a.x, row, a.B, a.C);
  const T* rr = a.has_res ? row_ptr<T>(a.r, row, a.B, a.C) : nullptr;
  float sumsq = 0.f;
  for (int64_t j = threadIdx.x; j < a.n; j += blockDim.x) {
    float s = to_f32(xr[j * a.x.col]);
    if (a.has_res) s += to_f32(rr[j * a.r.col]);
    sumsq += s * s;
  }
  sumsq = warp_sum(sumsq);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sumsq;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) tot += red[w];
  const float inv = rsqrtf(tot / static_cast<float>(a.n) + a.eps);
  T* yr = row_ptr<T>(a.y, row, a.B, a.C);
  T* ror = a.store_res ? row_ptr<T>(a.ro, row, a.B, a.C) : nullptr;
  for (int64_t j = threadIdx.x; j < a.n; j += blockDim.x) {
    float s = to_f32(xr[j * a.x.col]);
    if (a.has_res) s += to_f32(rr[j * a.r.col]);
    if (a.store_res) ror[j * a.ro.col] = from_f32<T>(s);
    const float w = load_as_f32(a.w, a.w_dtype, j * a.w_stride);
    yr[j * a.y.col] = from_f32<T>(s * inv * w);
  }
}

template <typename T, int VPT, bool FLAT>
cudaError_t launch_rms_vec2(const RmsArgs& a, bool has_res, bool store_res, cudaStream_t st) {
  const dim3 threads(32 * a.wpr * a.rpc);
  const dim3 blocks(static_cast<unsigned>((a.rows + a.rpc - 1) / a.rpc));
  using fd_host::launch_pdl;
  if (has_res && store_res) return launch_pdl(rms_vec_kernel<T, VPT, true, true, FLAT>, blocks, threads, 0, st, a);
  if (has_res) return launch_pdl(rms_vec_kernel<T, VPT, true, false, FLAT>, blocks, threads, 0, st, a);
  if (store_res) return launch_pdl(rms_vec_kernel<T, VPT, false, true, FLAT>, blocks, threads, 0, st, a);
  return launch_pdl(rms_vec_kernel<T, VPT, false, false, FLAT>, blocks, threads, 0, st, a);
}

template <typename T, int VPT>
cudaError_t launch_rms_vec(const RmsArgs& a, bool has_res, bool store_res, cudaStream_t st) {
  return a.flat ? launch_rms_vec2<T, VPT, true>(a, has_res, store_res, st)
                : launch_rms_vec2<T, VPT, false>(a, has_res, store_res, st);
}

template <typename T>
cudaError_t dispatch_rms_vec(RmsArgs& a, bool has_res, bool store_res, cudaStream_t st) {
  // Choose vectors-per-thread and warps-per-row so that a row stays in
  // registers: short rows pack several rows into one 128-thread CTA.
  const int nv = a.nv;
  if (nv <= 32) {
    a.wpr = 1; a.rpc = 4;
    return launch_rms_vec<T, 1>(a, has_res, store_res, st);
  }
  if (nv <= 64) {
    a.wpr = 1; a.rpc = 4;
    return launch_rms_vec<T, 2>(a, has_res, store_res, st);
  }
  a.rpc = 1;
  int wpr = (nv + 32 * 4 - 1) / (32 * 4);
  if (wpr <= 16) {
    a.wpr = wpr;
    return launch_rms_vec<T, 4>(a, has_res, store_res, st);
  }
  wpr = (nv + 32 * 8 - 1) / (32 * 8);
  a.wpr = wpr;  // <= 16 guaranteed by the caller (n <= 32768)
  return launch_rms_vec<T, 8>(a, has_res, store_res, st);
}

// ============================================================== SwiGLU
struct SwigluArgs {
  RowsArg g, u, y;
  int64_t B, C, rows;
  int64_t n;
  int64_t nv;     // vectors per row (vector path)
  int64_t items;  // rows * nv (vector path) or rows * n (scalar path)
};

// I is the index type of the item -> (row, vector) split: 32-bit whenever the
// item count fits, which keeps the per-item divisions cheap.
template <typename T, bool FLAT, typename I>
__global__ void __launch_bounds__(256) swiglu_vec_kernel(SwigluArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const I stride = static_cast<I>(gridDim.x) * blockDim.x;
  const I items = static_cast<I>(a.items), nv = static_cast<I>(a.nv);
  for (I it = static_cast<I>(blockIdx.x) * blockDim.x + threadIdx.x; it < items; it += stride) {
    const I row = it / nv;
    const int64_t j = it - row * nv;
    int64_t og, ou, oy;
    if (FLAT) {
      og = static_cast<int64_t>(row) * a.g.sc; ou = static_cast<int64_t>(row) * a.u.sc;
      oy = static_cast<int64_t>(row) * a.y.sc;
    } else {
      const I C = static_cast<I>(a.C), B = static_cast<I>(a.B);
      const I ic = row % C, t = row / C, ib = t % B, ia = t / B;
      og = ia * a.g.sa + ib * a.g.sb + ic * a.g.sc;
      ou = ia * a.u.sa + ib * a.u.sb + ic * a.u.sc;
      oy = ia * a.y.sa + ib * a.y.sb + ic * a.y.sc;
    }
    const uint4 gv = ld_stream16(reinterpret_cast<const T*>(a.g.ptr) + og + 8 * j);
    const uint4 uv = ld_stream16(reinterpret_cast<const T*>(a.u.ptr) + ou + 8 * j);
    float gf[8], uf[8], o[8];
    unpack8<T>(gv, gf);
    unpack8<T>(uv, uf);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = silu_mul(gf[e], uf[e]);
    st_stream16(reinterpret_cast<T*>(a.y.ptr) + oy + 8 * j, pack8<T>(o));
  }
}

template <typename T>
__global__ void __launch_bounds__(256) swiglu_generic_kernel(SwigluArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t it = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; it < a.items;
       it += stride) {
    const int64_t row = it / a.n;
    const int64_t j = it - row * a.n;
    const T* gp = row_ptr<T>(a.g, row, a.B, a.C);
    const T* up = row_ptr<T>(a.u, row, a.B, a.C);
    T* yp = row_ptr<T>(a.y, row, a.B, a.C);
    yp[j * a.y.col] = from_f32<T>(silu_mul(to_f32(gp[j * a.g.col]), to_f32(up[j * a.u.col])));
  }
}

unsigned fill_blocks(const void* kernel, int64_t items, int threads);
bool narrow_items(int64_t items);

// A grid-stride kernel over a.items, one full wave of CTAs, PDL launch.
template <typename Args>
cudaError_t launch_stream(void (*kernel)(Args), const Args& a, int64_t items, cudaStream_t st) {
  const unsigned blocks = fill_blocks(reinterpret_cast<const void*>(kernel), items, 256);
  return fd_host::launch_pdl(kernel, blocks, 256, 0, st, a);
}

template <typename T>
cudaError_t launch_swiglu_vec(const SwigluArgs& a, bool flat, cudaStream_t st) {
  const bool narrow = narrow_items(a.items);
  if (flat && narrow) return launch_stream(swiglu_vec_kernel<T, true, uint32_t>, a, a.items, st);
  if (flat) return launch_stream(swiglu_vec_kernel<T, true, int64_t>, a, a.items, st);
  if (narrow) return launch_stream(swiglu_vec_kernel<T, false, uint32_t>, a, a.items, st);
  return launch_stream(swiglu_vec_kernel<T, false, int64_t>, a, a.items, st);
}

// ============================================================== RoPE
struct RopeArgs {
  RowsArg x, c, s, y;
  int32_t c_dtype, s_dtype;
  int64_t B, C, rows;
  int64_t half;
  int64_t hv;     // 8-element vectors per half row (vector path)
  int64_t items;
};

// Eight RoPE angles (cos or sin) of element type CT, kept packed until used.
template <typename CT>
struct Angles8 {
  uint4 v;
  FD_DEV void load(const CT* p) { v = __ldg(reinterpret_cast<const uint4*>(p)); }
  FD_DEV float2 pair(int w) const { return unpack2<CT>(w == 0 ? v.x : w == 1 ? v.y : w == 2 ? v.z : v.w); }
};
template <>
struct Angles8<float> {
  float4 lo, hi;
  FD_DEV void load(const float* p) {
    lo = __ldg(reinterpret_cast<const float4*>(p));
    hi = __ldg(reinterpret_cast<const float4*>(p) + 1);
  }
  FD_DEV float2 pair(int w) const {
    return w == 0 ? make_float2(lo.x, lo.y) : w == 1 ? make_float2(lo.z, lo.w)
         : w == 2 ? make_float2(hi.x, hi.y) : make_float2(hi.z, hi.w);
  }
};

// Vector path: one item = 8 elements of each half of one row.  CT is the
// element type of cos and sin (one type for both here).
template <typename T, typename CT, typename I>
__global__ void __launch_bounds__(256) rope_vec_kernel(RopeArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const I stride = static_cast<I>(gridDim.x) * blockDim.x;
  const I items = static_cast<I>(a.items), hv = static_cast<I>(a.hv);
  const I C = static_cast<I>(a.C), B = static_cast<I>(a.B);
  for (I it = static_cast<I>(blockIdx.x) * blockDim.x + threadIdx.x; it < items; it += stride) {
    const I row = it / hv;
    const int64_t j = 8 * static_cast<int64_t>(it - row * hv);
    const I ic = row % C, tt = row / C, ib = tt % B, ia = tt / B;
    const T* xp = reinterpret_cast<const T*>(a.x.ptr) + (ia * a.x.sa + ib * a.x.sb + ic * a.x.sc);
    const CT* cp = reinterpret_cast<const CT*>(a.c.ptr) + (ia * a.c.sa + ib * a.c.sb + ic * a.c.sc);
    const CT* sp = reinterpret_cast<const CT*>(a.s.ptr) + (ia * a.s.sa + ib * a.s.sb + ic * a.s.sc);
    T* yp = reinterpret_cast<T*>(a.y.ptr) + (ia * a.y.sa + ib * a.y.sb + ic * a.y.sc);
    const uint4 x1 = ld_stream16(xp + j);
    const uint4 x2 = ld_stream16(xp + a.half + j);
    Angles8<CT> c1, c2, s1, s2;
    c1.load(cp + j);
    c2.load(cp + a.half + j);
    s1.load(sp + j);
    s2.load(sp + a.half + j);
    const uint32_t xw1[4] = {x1.x, x1.y, x1.z, x1.w}, xw2[4] = {x2.x, x2.y, x2.z, x2.w};
    uint32_t o1[4], o2[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float2 a1 = unpack2<T>(xw1[w]), a2 = unpack2<T>(xw2[w]);
      const float2 cc1 = c1.pair(w), cc2 = c2.pair(w), ss1 = s1.pair(w), ss2 = s2.pair(w);
      o1[w] = pack2<T>(a1.x * cc1.x - a2.x * ss1.x, a1.y * cc1.y - a2.y * ss1.y);
      o2[w] = pack2<T>(a2.x * cc2.x + a1.x * ss2.x, a2.y * cc2.y + a1.y * ss2.y);
    }
    st_stream16(yp + j, make_uint4(o1[0], o1[1], o1[2], o1[3]));
    st_stream16(yp + a.half + j, make_uint4(o2[0], o2[1], o2[2], o2[3]));
  }
}

template <typename T>
__global__ void __launch_bounds__(256) rope_generic_kernel(RopeArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t it = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; it < a.items;
       it += stride) {
    const int64_t row = it / a.half;
    const int64_t j = it - row * a.half;
    const T* xp = row_ptr<T>(a.x, row, a.B, a.C);
    T* yp = row_ptr<T>(a.y, row, a.B, a.C);
    const int64_t oc = row_base(row, a.B, a.C, a.c.sa, a.c.sb, a.c.sc);
    const int64_t os = row_base(row, a.B, a.C, a.s.sa, a.s.sb, a.s.sc);
    const float x1 = to_f32(xp[j * a.x.col]);
    const float x2 = to_f32(xp[(j + a.half) * a.x.col]);
    const float c1 = load_as_f32(a.c.ptr, a.c_dtype, oc + j * a.c.col);
    const float c2 = load_as_f32(a.c.ptr, a.c_dtype, oc + (j + a.half) * a.c.col);
    const float s1 = load_as_f32(a.s.ptr, a.s_dtype, os + j * a.s.col);
    const float s2 = load_as_f32(a.s.ptr, a.s_dtype, os + (j + a.half) * a.s.col);
    yp[j * a.y.col] = from_f32<T>(x1 * c1 - x2 * s1);
    yp[(j + a.half) * a.y.col] = from_f32<T>(x2 * c2 + x1 * s2);
  }
}

template <typename T, typename CT>
cudaError_t launch_rope_vec2(const RopeArgs& a, cudaStream_t st) {
  return narrow_items(a.items) ? launch_stream(rope_vec_kernel<T, CT, uint32_t>, a, a.items, st)
                               : launch_stream(rope_vec_kernel<T, CT, int64_t>, a, a.items, st);
}
template <typename T>
cudaError_t launch_rope_vec(const RopeArgs& a, int cs_dtype, cudaStream_t st) {
  if (cs_dtype == FD_F32) return launch_rope_vec2<T, float>(a, st);
  if (cs_dtype == FD_BF16) return launch_rope_vec2<T, __nv_bfloat16>(a, st);
  return launch_rope_vec2<T, __half>(a, st);
}

// ============================================================== copy / triad
__global__ void __launch_bounds__(256) copy_vec_kernel(uint4* __restrict__ dst,
                                                       const uint4* __restrict__ src, int64_t nv) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  // Four independent 16-byte loads in flight per thread per iteration.
  for (; i + 3 * stride < nv; i += 4 * stride) {
    const uint4 v0 = ld_stream16(src + i);
    const uint4 v1 = ld_stream16(src + i + stride);
    const uint4 v2 = ld_stream16(src + i + 2 * stride);
    const uint4 v3 = ld_stream16(src + i + 3 * stride);
    st_stream16(dst + i, v0);
    st_stream16(dst + i + stride, v1);
    st_stream16(dst + i + 2 * stride, v2);
    st_stream16(dst + i + 3 * stride, v3);
  }
  for (; i < nv; i += stride) st_stream16(dst + i, ld_stream16(src + i));
}

__global__ void copy_bytes_kernel(char* __restrict__ dst, const char* __restrict__ src, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = src[i];
}

template <typename T>
__global__ void __launch_bounds__(256) triad_vec_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                                        T* __restrict__ c, int64_t nv, float scale) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nv; i += stride) {
    float af[8], bf[8], o[8];
    unpack8<T>(ld_stream16(a + 8 * i), af);
    unpack8<T>(ld_stream16(b + 8 * i), bf);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = af[e] + bf[e] * scale;
    st_stream16(c + 8 * i, pack8<T>(o));
  }
}

template <typename T>
__global__ void triad_scalar_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ c,
                                    int64_t n, float scale) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    c[i] = from_f32<T>(to_f32(a[i]) + to_f32(b[i]) * scale);
}

// out = round(partial + residual): the residual add that follows the
// tensor-parallel allreduce of fp32 down-projection partials.
template <typename T>
__global__ void __launch_bounds__(256) residual_add_kernel(const float* __restrict__ partial,
                                                           const T* __restrict__ res, T* __restrict__ out,
                                                           int64_t n) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = from_f32<T>(partial[i] + to_f32(res[i]));
}

// CTAs of `threads` threads for a grid-stride kernel over `items`: as many as
// are resident at once (one full wave, no tail wave), fewer for small inputs.
unsigned fill_blocks(const void* kernel, int64_t items, int threads) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> per_sm;
  int occ = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = per_sm.find(kernel);
    if (it == per_sm.end()) {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, 0) != cudaSuccess || occ < 1) occ = 1;
      per_sm.emplace(kernel, occ);
    } else {
      occ = it->second;
    }
  }
  const int64_t cap = static_cast<int64_t>(fd_host::sm_count()) * occ;
  const int64_t need = std::max<int64_t>(1, (items + threads - 1) / threads);
  return static_cast<unsigned>(std::min(need, cap));
}

// True when a 32-bit grid-stride index over `items` cannot overflow.
bool narrow_items(int64_t items) { return items + static_cast<int64_t>(fd_host::sm_count()) * 2048 < (int64_t{1} << 32); }

unsigned stream_blocks(int64_t items, int threads) {
  // Enough CTAs to fill every SM with 2048 threads, grid-striding beyond that.
  const int64_t cap = static_cast<int64_t>(fd_host::sm_count()) * (2048 / threads);
  int64_t need = (items + threads - 1) / threads;
  if (need < 1) need = 1;
  return static_cast<unsigned>(std::min(need, cap));
}

int from_cuda(cudaError_t e) { return e == cudaSuccess ? FD_OK : FD_ERR_LAUNCH; }

}  // namespace

namespace fd_host {

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace fd_host

// ================================================================ C ABI
extern "C" {

const char* fd_status_string(int status) {
  switch (status) {
    case FD_OK: return "ok";
    case FD_ERR_ARG: return "invalid argument";
    case FD_ERR_LAUNCH: return "kernel launch failed";
    case FD_ERR_WORKSPACE: return "workspace missing or too small";
    case FD_ERR_UNSUPPORTED: return "unsupported shape";
    case FD_ERR_DEVICE: return "device query failed";
    default: return "unknown status";
  }
}

int fd_device_sm_count(void) { return fd_host::sm_count(); }

int fd_rms_out(const fd_rows* x, const fd_rows* residual, const void* weight, int32_t w_dtype,
               int64_t w_stride, const fd_rows* out, const fd_rows* residual_out, float eps,
               void* stream) {
  using namespace fd_host;
  if (!x || !out || !weight) return FD_ERR_ARG;
  if (!half_dtype(x->dtype) || out->dtype != x->dtype || !valid_dtype(w_dtype)) return FD_ERR_ARG;
  if (!same_grid(x, out)) return FD_ERR_ARG;
  const bool has_res = residual != nullptr;
  const bool store_res = residual_out != nullptr;
  if (has_res && (!same_grid(x, residual) || residual->dtype != x->dtype)) return FD_ERR_ARG;
  if (store_res && (!same_grid(x, residual_out) || residual_out->dtype != x->dtype)) return FD_ERR_ARG;
  const int64_t rows = x->a * x->b * x->c;
  if (rows <= 0 || x->n <= 0) return FD_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf = x->dtype == FD_BF16;

  const bool vec = (x->n % 8 == 0) && x->n <= 32768 && rows < (int64_t{1} << 31) && rows_vec16(x) &&
                   rows_vec16(out) && (!has_res || rows_vec16(residual)) &&
                   (!store_res || rows_vec16(residual_out)) && w_stride == 1 && aligned16(weight);
  if (vec) {
    RmsArgs a;
    a.x = rows_arg(x); a.r = rows_arg(has_res ? residual : x);
    a.y = rows_arg(out); a.ro = rows_arg(store_res ? residual_out : out);
    a.B = x->b; a.C = x->c; a.rows = rows;
    a.w = weight; a.w_dtype = w_dtype;
    a.nv = static_cast<int32_t>(x->n / 8); a.n = static_cast<int32_t>(x->n);
    a.eps = eps; a.wpr = 1; a.rpc = 1;
    a.flat = x->a == 1 && x->b == 1;
    cudaError_t e = bf ? dispatch_rms_vec<__nv_bfloat16>(a, has_res, store_res, st)
                       : dispatch_rms_vec<__half>(a, has_res, store_res, st);
    return from_cuda(e);
  }
  RmsGenArgs g;
  g.x = rows_arg(x); g.r = rows_arg(has_res ? residual : x);
  g.y = rows_arg(out); g.ro = rows_arg(store_res ? residual_out : out);
  g.B = x->b; g.C = x->c; g.rows = rows;
  g.w = weight; g.w_dtype = w_dtype; g.w_stride = w_stride;
  g.n = x->n; g.eps = eps; g.has_res = has_res; g.store_res = store_res;
  if (rows > 0x7fffffffLL) return FD_ERR_UNSUPPORTED;
  using fd_host::launch_pdl;
  const dim3 blocks(static_cast<unsigned>(rows));
  const cudaError_t e = bf ? launch_pdl(rms_generic_kernel<__nv_bfloat16>, blocks, 256, 0, st, g)
                           : launch_pdl(rms_generic_kernel<__half>, blocks, 256, 0, st, g);
  return from_cuda(e);
}

int fd_swiglu_out(const fd_rows* gate, const fd_rows* up, const fd_rows* out, void* stream) {
  using namespace fd_host;
  if (!gate || !up || !out) return FD_ERR_ARG;
  if (!half_dtype(gate->dtype) || up->dtype != gate->dtype || out->dtype != gate->dtype) return FD_ERR_ARG;
  if (!same_grid(gate, up) || !same_grid(gate, out)) return FD_ERR_ARG;
  const int64_t rows = gate->a * gate->b * gate->c;
  if (rows <= 0 || gate->n <= 0) return FD_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf = gate->dtype == FD_BF16;
  SwigluArgs a;
  a.g = rows_arg(gate); a.u = rows_arg(up); a.y = rows_arg(out);
  a.B = gate->b; a.C = gate->c; a.rows = rows; a.n = gate->n;
  const bool vec = gate->n % 8 == 0 && rows_vec16(gate) && rows_vec16(up) && rows_vec16(out);
  if (vec) {
    a.nv = gate->n / 8;
    a.items = rows * a.nv;
    const bool flat = gate->a == 1 && gate->b == 1;
    const cudaError_t e = bf ? launch_swiglu_vec<__nv_bfloat16>(a, flat, st) : launch_swiglu_vec<__half>(a, flat, st);
    return from_cuda(e);
  }
  a.nv = 0;
  a.items = rows * gate->n;
  const cudaError_t e = bf ? launch_stream(swiglu_generic_kernel<__nv_bfloat16>, a, a.items, st)
                           : launch_stream(swiglu_generic_kernel<__half>, a, a.items, st);
  return from_cuda(e);
}

int fd_rope_out(const fd_rows* x, const fd_rows* cos, const fd_rows* sin, const fd_rows* out,
                void* stream) {
  using namespace fd_host;
  if (!x || !cos || !sin || !out) return FD_ERR_ARG;
  if (!half_dtype(x->dtype) || out->dtype != x->dtype) return FD_ERR_ARG;
  if (!valid_dtype(cos->dtype) || !valid_dtype(sin->dtype)) return FD_ERR_ARG;
  if (!same_grid(x, cos) || !same_grid(x, sin) || !same_grid(x, out)) return FD_ERR_ARG;
  if (x->n % 2 != 0) return FD_ERR_ARG;
  const int64_t rows = x->a * x->b * x->c;
  if (rows <= 0 || x->n <= 0) return FD_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf = x->dtype == FD_BF16;
  RopeArgs a;
  a.x = rows_arg(x); a.c = rows_arg(cos); a.s = rows_arg(sin); a.y = rows_arg(out);
  a.c_dtype = cos->dtype; a.s_dtype = sin->dtype;
  a.B = x->b; a.C = x->c; a.rows = rows;
  a.half = x->n / 2;
  const bool vec = a.half % 8 == 0 && cos->dtype == sin->dtype && rows_vec16(x) && rows_vec16(cos) &&
                   rows_vec16(sin) && rows_vec16(out);
  if (vec) {
    a.hv = a.half / 8;
    a.items = rows * a.hv;
    const cudaError_t e = bf ? launch_rope_vec<__nv_bfloat16>(a, cos->dtype, st)
                             : launch_rope_vec<__half>(a, cos->dtype, st);
    return from_cuda(e);
  }
  a.hv = 0;
  a.items = rows * a.half;
  const cudaError_t e = bf ? launch_stream(rope_generic_kernel<__nv_bfloat16>, a, a.items, st)
                           : launch_stream(rope_generic_kernel<__half>, a, a.items, st);
  return from_cuda(e);
}

int fd_residual_add_out(const float* partial, const void* residual, void* out, int32_t dtype, int64_t n,
                        void* stream) {
  using namespace fd_host;
  if (n == 0) return FD_OK;
  if (!partial || !residual || !out || n < 0 || !half_dtype(dtype)) return FD_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned blocks = stream_blocks(n, 256);
  using fd_host::launch_pdl;
  const cudaError_t e =
      dtype == FD_BF16
          ? launch_pdl(residual_add_kernel<__nv_bfloat16>, blocks, 256, 0, st, partial,
                       static_cast<const __nv_bfloat16*>(residual), static_cast<__nv_bfloat16*>(out), n)
          : launch_pdl(residual_add_kernel<__half>, blocks, 256, 0, st, partial, static_cast<const __half*>(residual),
                       static_cast<__half*>(out), n);
  return from_cuda(e);
}

int fd_copy(void* dst, const void* src, size_t bytes, void* stream) {
  using namespace fd_host;
  if (bytes == 0) return FD_OK;
  if (!dst || !src) return FD_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (aligned16(dst) && aligned16(src)) {
    const int64_t nv = static_cast<int64_t>(bytes / 16);
    if (nv > 0) {
      copy_vec_kernel<<<stream_blocks(nv, 256), 256, 0, st>>>(static_cast<uint4*>(dst),
                                                              static_cast<const uint4*>(src), nv);
    }
    const int64_t tail = static_cast<int64_t>(bytes % 16);
    if (tail) {
      copy_bytes_kernel<<<1, 32, 0, st>>>(static_cast<char*>(dst) + nv * 16,
                                          static_cast<const char*>(src) + nv * 16, tail);
    }
    return from_cuda(cudaGetLastError());
  }
  copy_bytes_kernel<<<stream_blocks(static_cast<int64_t>(bytes), 256), 256, 0, st>>>(
      static_cast<char*>(dst), static_cast<const char*>(src), static_cast<int64_t>(bytes));
  return from_cuda(cudaGetLastError());
}

int fd_triad(const void* a, const void* b, void* c, int64_t n, int32_t dtype, float scale, void* stream) {
  using namespace fd_host;
  if (n == 0) return FD_OK;
  if (!a || !b || !c || n < 0 || !valid_dtype(dtype)) return FD_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool vec = dtype != FD_F32 && n % 8 == 0 && aligned16(a) && aligned16(b) && aligned16(c);
  if (vec) {
    const int64_t nv = n / 8;
    const unsigned blocks = stream_blocks(nv, 256);
    if (dtype == FD_BF16)
      triad_vec_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
          static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b),
          static_cast<__nv_bfloat16*>(c), nv, scale);
    else
      triad_vec_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<const __half*>(a),
                                                       static_cast<const __half*>(b),
                                                       static_cast<__half*>(c), nv, scale);
    return from_cuda(cudaGetLastError());
  }
  const unsigned blocks = stream_blocks(n, 256);
  if (dtype == FD_BF16)
    triad_scalar_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b),
        static_cast<__nv_bfloat16*>(c), n, scale);
  else if (dtype == FD_F16)
    triad_scalar_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<const __half*>(a),
                                                        static_cast<const __half*>(b),
                                                        static_cast<__half*>(c), n, scale);
  else
    triad_scalar_kernel<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(a),
                                                       static_cast<const float*>(b),
                                                       static_cast<float*>(c), n, scale);
  return from_cuda(cudaGetLastError());
}

}  // extern "C"
