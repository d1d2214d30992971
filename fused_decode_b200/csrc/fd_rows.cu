// Row-wise and elementwise decode kernels for sm_100a:
//   RMSNorm / fused add+RMSNorm, SwiGLU, rotate-half RoPE, and the copy / triad
//   roof kernels.  All are HBM-streaming kernels: 16-byte vector loads and
//   stores, fp32 math, one rounding to the activation dtype per output, and a
//   scalar fallback for any layout the vector path cannot address.
#include "fd_common.cuh"

#include <algorithm>

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
  const void* w;
  int32_t w_dtype;
  int32_t wpr;   // warps per row
  int32_t rpc;   // rows per CTA
  int32_t nv;    // vectors (8 elements) per row
  int32_t n;
  float eps;
};

template <typename T, int VPT, bool HAS_RES, bool STORE_RES>
__global__ void __launch_bounds__(512) rms_vec_kernel(RmsArgs a) {
  __shared__ float red[32];
  const int group_threads = 32 * a.wpr;
  const int group = threadIdx.x / group_threads;
  const int t = threadIdx.x - group * group_threads;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * a.rpc + group;
  const bool live = row < a.rows;

  float s[VPT][8];
  float sumsq = 0.f;
  if (live) {
    const T* xr = row_ptr<T>(a.x, row, a.B, a.C);
    const T* rr = HAS_RES ? row_ptr<T>(a.r, row, a.B, a.C) : nullptr;
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
      T* ror = row_ptr<T>(a.ro, row, a.B, a.C);
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
  const float inv = 1.0f / sqrtf(sumsq / static_cast<float>(a.n) + a.eps);
  T* yr = row_ptr<T>(a.y, row, a.B, a.C);
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
  const float inv = 1.0f / sqrtf(tot / static_cast<float>(a.n) + a.eps);
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

template <typename T, int VPT>
cudaError_t launch_rms_vec(const RmsArgs& a, bool has_res, bool store_res, cudaStream_t st) {
  const int threads = 32 * a.wpr * a.rpc;
  const unsigned blocks = static_cast<unsigned>((a.rows + a.rpc - 1) / a.rpc);
  if (has_res && store_res)
    rms_vec_kernel<T, VPT, true, true><<<blocks, threads, 0, st>>>(a);
  else if (has_res)
    rms_vec_kernel<T, VPT, true, false><<<blocks, threads, 0, st>>>(a);
  else if (store_res)
    rms_vec_kernel<T, VPT, false, true><<<blocks, threads, 0, st>>>(a);
  else
    rms_vec_kernel<T, VPT, false, false><<<blocks, threads, 0, st>>>(a);
  return cudaGetLastError();
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

FD_DEV float silu_mul(float g, float u) {
  // Stable sigmoid, as the reference kernel computes it (kernels.py:448-451).
  const float e = expf(-fabsf(g));
  const float sig = g >= 0.f ? 1.0f / (1.0f + e) : e / (1.0f + e);
  return g * sig * u;
}

template <typename T, bool FLAT>
__global__ void __launch_bounds__(256) swiglu_vec_kernel(SwigluArgs a) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t it = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; it < a.items;
       it += stride) {
    const int64_t row = it / a.nv;
    const int64_t j = it - row * a.nv;
    int64_t og, ou, oy;
    if (FLAT) {
      og = row * a.g.sc; ou = row * a.u.sc; oy = row * a.y.sc;
    } else {
      og = row_base(row, a.B, a.C, a.g.sa, a.g.sb, a.g.sc);
      ou = row_base(row, a.B, a.C, a.u.sa, a.u.sb, a.u.sc);
      oy = row_base(row, a.B, a.C, a.y.sa, a.y.sb, a.y.sc);
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

// ============================================================== RoPE
struct RopeArgs {
  RowsArg x, c, s, y;
  int32_t c_dtype, s_dtype;
  int64_t B, C, rows;
  int64_t half;
  int64_t hv;     // 8-element vectors per half row (vector path)
  int64_t items;
};

template <typename T>
__global__ void __launch_bounds__(256) rope_vec_kernel(RopeArgs a) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int ces = a.c_dtype == FD_F32 ? 4 : 2;
  const int ses = a.s_dtype == FD_F32 ? 4 : 2;
  for (int64_t it = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; it < a.items;
       it += stride) {
    const int64_t row = it / a.hv;
    const int64_t j = 8 * (it - row * a.hv);
    const int64_t ic = row % a.C;
    const int64_t tt = row / a.C;
    const int64_t ib = tt % a.B;
    const int64_t ia = tt / a.B;
    const int64_t ox = ia * a.x.sa + ib * a.x.sb + ic * a.x.sc;
    const int64_t oc = ia * a.c.sa + ib * a.c.sb + ic * a.c.sc;
    const int64_t os = ia * a.s.sa + ib * a.s.sb + ic * a.s.sc;
    const int64_t oy = ia * a.y.sa + ib * a.y.sb + ic * a.y.sc;
    const T* xp = reinterpret_cast<const T*>(a.x.ptr) + ox;
    float x1[8], x2[8], c1[8], c2[8], s1[8], s2[8];
    unpack8<T>(ld_stream16(xp + j), x1);
    unpack8<T>(ld_stream16(xp + a.half + j), x2);
    load8_as_f32(a.c.ptr + (oc + j) * ces, a.c_dtype, c1);
    load8_as_f32(a.c.ptr + (oc + a.half + j) * ces, a.c_dtype, c2);
    load8_as_f32(a.s.ptr + (os + j) * ses, a.s_dtype, s1);
    load8_as_f32(a.s.ptr + (os + a.half + j) * ses, a.s_dtype, s2);
    float o1[8], o2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o1[e] = x1[e] * c1[e] - x2[e] * s1[e];
      o2[e] = x2[e] * c2[e] + x1[e] * s2[e];
    }
    T* yp = reinterpret_cast<T*>(a.y.ptr) + oy;
    st_stream16(yp + j, pack8<T>(o1));
    st_stream16(yp + a.half + j, pack8<T>(o2));
  }
}

template <typename T>
__global__ void __launch_bounds__(256) rope_generic_kernel(RopeArgs a) {
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
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = from_f32<T>(partial[i] + to_f32(res[i]));
}

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

  const bool vec = (x->n % 8 == 0) && x->n <= 32768 && rows_vec16(x) && rows_vec16(out) &&
                   (!has_res || rows_vec16(residual)) && (!store_res || rows_vec16(residual_out)) &&
                   w_stride == 1 && aligned16(weight);
  if (vec) {
    RmsArgs a;
    a.x = rows_arg(x); a.r = rows_arg(has_res ? residual : x);
    a.y = rows_arg(out); a.ro = rows_arg(store_res ? residual_out : out);
    a.B = x->b; a.C = x->c; a.rows = rows;
    a.w = weight; a.w_dtype = w_dtype;
    a.nv = static_cast<int32_t>(x->n / 8); a.n = static_cast<int32_t>(x->n);
    a.eps = eps; a.wpr = 1; a.rpc = 1;
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
  if (bf)
    rms_generic_kernel<__nv_bfloat16><<<static_cast<unsigned>(rows), 256, 0, st>>>(g);
  else
    rms_generic_kernel<__half><<<static_cast<unsigned>(rows), 256, 0, st>>>(g);
  return from_cuda(cudaGetLastError());
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
    const unsigned blocks = stream_blocks(a.items, 256);
    if (bf) {
      if (flat) swiglu_vec_kernel<__nv_bfloat16, true><<<blocks, 256, 0, st>>>(a);
      else swiglu_vec_kernel<__nv_bfloat16, false><<<blocks, 256, 0, st>>>(a);
    } else {
      if (flat) swiglu_vec_kernel<__half, true><<<blocks, 256, 0, st>>>(a);
      else swiglu_vec_kernel<__half, false><<<blocks, 256, 0, st>>>(a);
    }
    return from_cuda(cudaGetLastError());
  }
  a.nv = 0;
  a.items = rows * gate->n;
  const unsigned blocks = stream_blocks(a.items, 256);
  if (bf) swiglu_generic_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(a);
  else swiglu_generic_kernel<__half><<<blocks, 256, 0, st>>>(a);
  return from_cuda(cudaGetLastError());
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
  const bool vec = a.half % 8 == 0 && rows_vec16(x) && rows_vec16(cos) && rows_vec16(sin) &&
                   rows_vec16(out);
  if (vec) {
    a.hv = a.half / 8;
    a.items = rows * a.hv;
    const unsigned blocks = stream_blocks(a.items, 256);
    if (bf) rope_vec_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(a);
    else rope_vec_kernel<__half><<<blocks, 256, 0, st>>>(a);
    return from_cuda(cudaGetLastError());
  }
  a.hv = 0;
  a.items = rows * a.half;
  const unsigned blocks = stream_blocks(a.items, 256);
  if (bf) rope_generic_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(a);
  else rope_generic_kernel<__half><<<blocks, 256, 0, st>>>(a);
  return from_cuda(cudaGetLastError());
}

int fd_residual_add_out(const float* partial, const void* residual, void* out, int32_t dtype, int64_t n,
                        void* stream) {
  using namespace fd_host;
  if (n == 0) return FD_OK;
  if (!partial || !residual || !out || n < 0 || !half_dtype(dtype)) return FD_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned blocks = stream_blocks(n, 256);
  if (dtype == FD_BF16)
    residual_add_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        partial, static_cast<const __nv_bfloat16*>(residual), static_cast<__nv_bfloat16*>(out), n);
  else
    residual_add_kernel<__half><<<blocks, 256, 0, st>>>(partial, static_cast<const __half*>(residual),
                                                        static_cast<__half*>(out), n);
  return from_cuda(cudaGetLastError());
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
