// Shared device helpers for the sm_100a decode kernels: element conversion,
// 16-byte vector access, row addressing and warp reductions.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/fd_b200.h"

#define FD_DEV __device__ __forceinline__

namespace fd {

// ---------------------------------------------------------------- conversion
FD_DEV float to_f32(__half v) { return __half2float(v); }
FD_DEV float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
FD_DEV float to_f32(float v) { return v; }

template <typename T>
FD_DEV T from_f32(float v);
template <>
FD_DEV __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
FD_DEV __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
FD_DEV float from_f32<float>(float v) { return v; }

// Round an fp32 value to T and back (the reference's `.to(dtype)` points).
template <typename T>
FD_DEV float round_to(float v) { return to_f32(from_f32<T>(v)); }

// Two packed 16-bit values in one 32-bit word -> two floats.
template <typename T>
FD_DEV float2 unpack2(uint32_t w);
template <>
FD_DEV float2 unpack2<__half>(uint32_t w) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  return __half22float2(h);
}
template <>
FD_DEV float2 unpack2<__nv_bfloat16>(uint32_t w) {
  // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32 word.
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

template <typename T>
FD_DEV uint32_t pack2(float a, float b);
template <>
FD_DEV uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
FD_DEV uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// 8 packed 16-bit elements (one uint4) <-> 8 floats.
template <typename T>
FD_DEV void unpack8(const uint4& v, float* f) {
  float2 p;
  p = unpack2<T>(v.x); f[0] = p.x; f[1] = p.y;
  p = unpack2<T>(v.y); f[2] = p.x; f[3] = p.y;
  p = unpack2<T>(v.z); f[4] = p.x; f[5] = p.y;
  p = unpack2<T>(v.w); f[6] = p.x; f[7] = p.y;
}
template <typename T>
FD_DEV uint4 pack8(const float* f) {
  uint4 v;
  v.x = pack2<T>(f[0], f[1]);
  v.y = pack2<T>(f[2], f[3]);
  v.z = pack2<T>(f[4], f[5]);
  v.w = pack2<T>(f[6], f[7]);
  return v;
}

// Scalar load of element i of a runtime-typed array as fp32.
FD_DEV float load_as_f32(const void* p, int dtype, int64_t i) {
  if (dtype == FD_F32) return static_cast<const float*>(p)[i];
  if (dtype == FD_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

// As load_as_f32, but read through L2 only: for data another CTA may have
// written earlier in the same kernel.
FD_DEV float load_as_f32_cg(const void* p, int dtype, int64_t i) {
  if (dtype == FD_F32) return __ldcg(static_cast<const float*>(p) + i);
  const unsigned short bits = __ldcg(static_cast<const unsigned short*>(p) + i);
  if (dtype == FD_BF16) return __bfloat162float(__ushort_as_bfloat16(bits));
  return __half2float(__ushort_as_half(bits));
}

// 8 consecutive elements of a runtime-typed array as fp32 (16-byte aligned for
// 16-bit types, 32-byte region for f32 -- two 16-byte loads).
FD_DEV void load8_as_f32(const void* p, int dtype, float* f) {
  if (dtype == FD_F32) {
    const float4* q = static_cast<const float4*>(p);
    float4 a = __ldg(q), b = __ldg(q + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else if (dtype == FD_BF16) {
    unpack8<__nv_bfloat16>(__ldg(static_cast<const uint4*>(p)), f);
  } else {
    unpack8<__half>(__ldg(static_cast<const uint4*>(p)), f);
  }
}

// --------------------------------------------------------------- global I/O
// Streaming 16-byte load that does not allocate in L1 (data read once).
FD_DEV uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// Streaming 16-byte store (evict-first: written once, not re-read soon).
FD_DEV void st_stream16(void* p, const uint4& v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// ------------------------------------------------------------ row addressing
// Row r of an fd_rows grid -> element offset of its first element
// (the reference's _row_base, kernels.py:82-88).
struct RowGrid {
  int64_t b, c;          // sizes of the two inner leading dims
  int64_t sa, sb, sc;    // leading strides (elements)
  int64_t col;           // last-dim stride
};

FD_DEV int64_t row_base(int64_t row, int64_t B, int64_t C, int64_t sa, int64_t sb, int64_t sc) {
  int64_t c = row % C;
  int64_t t = row / C;
  int64_t b = t % B;
  int64_t a = t / B;
  return a * sa + b * sb + c * sc;
}

// silu(g) * u with the stable sigmoid of the reference kernel
// (kernels.py:448-451): e = exp(-|g|); sigmoid = 1/(1+e) for g >= 0, else
// e/(1+e).  exp and the reciprocal are the hardware approximations (__expf,
// __fdividef with a divisor in [1, 2]): a few fp32 ulp, far below the one
// rounding to the 16-bit output, and cheap enough that a streaming SwiGLU
// stays bound by HBM rather than by the IEEE divide.
FD_DEV float silu_mul(float g, float u) {
  const float e = __expf(-fabsf(g));
  const float r = __fdividef(1.0f, 1.0f + e);
  return g * (g >= 0.f ? r : e * r) * u;
}

// ------------------------------------------------- programmatic dependent launch
// Kernels launched with fd_host::launch_pdl may start while the previous
// kernel on the stream is still draining.  Every such kernel calls
// grid_dep_wait() before its first access to global memory another kernel may
// have written, and grid_dep_launch() once the next kernel may be scheduled.
FD_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
FD_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- reductions
FD_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace fd

// ------------------------------------------------- tensor-parallel exchange
// One rank's exchange buffer (device memory every rank of the group maps):
//   [header: round number, done counter; 256 B]
//   [data: 2 parities x world x m_max x n tagged words of 8 bytes]
// In round s rank r stores element (c, row) of its fp32 partial as the 8-byte
// word {value bits, s + 1} at data[s & 1][r][c][row] of every rank's buffer.
// An aligned 8-byte store arrives whole, so a reader that sees tag s + 1 also
// sees the value: no fence and no separate flag between writer and reader.
// Two parities let a rank run one round ahead of a slower peer without
// overwriting words the peer has not read yet (and a word left from round
// s - 2 carries tag s - 1).
constexpr int kMaxTpWorld = 8;
constexpr int kTpBlockRows = 128;
constexpr int kStatusTpTimeout = 8;  // status bit: a wait for a peer's word expired

// A tagged word as a peer stored it (an NVLink store into this buffer).
FD_DEV uint2 ld_tagged_sys(const uint2* p) {
  uint2 v;
  asm volatile("ld.relaxed.sys.global.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

struct TpLayout {
  int64_t nblk, data_off, bytes;
};

__host__ __device__ inline TpLayout tp_layout(int world, int m_max, int64_t n) {
  TpLayout l;
  l.nblk = (n + kTpBlockRows - 1) / kTpBlockRows;
  l.data_off = 256;
  l.bytes = l.data_off + 2LL * world * m_max * n * 8;
  return l;
}

// Host-side helpers shared by the entry points.
namespace fd_host {

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int elem_size(int dtype) { return dtype == FD_F32 ? 4 : 2; }

inline bool valid_dtype(int dtype) { return dtype == FD_F16 || dtype == FD_BF16 || dtype == FD_F32; }

inline bool half_dtype(int dtype) { return dtype == FD_F16 || dtype == FD_BF16; }

// True when every row of `r` starts on a 16-byte boundary and its elements are
// contiguous: the precondition of the 128-bit vector paths.
inline bool rows_vec16(const fd_rows* r) {
  if (r->col != 1) return false;
  const int64_t es = elem_size(r->dtype);
  if (!aligned16(r->ptr)) return false;
  // A leading stride only matters when its dimension has more than one index.
  if (r->a > 1 && ((r->sa * es) & 15)) return false;
  if (r->b > 1 && ((r->sb * es) & 15)) return false;
  if (r->c > 1 && ((r->sc * es) & 15)) return false;
  return true;
}

inline bool same_grid(const fd_rows* l, const fd_rows* r) {
  return l->a == r->a && l->b == r->b && l->c == r->c && l->n == r->n;
}

int sm_count();

// Finish a tensor-parallel MLP layer (fd_tp.cu): out = round(sum of the
// ranks' partials in `buf` + res), once every word carries the round's tag.
int tp_reduce_launch(char* buf, int world, int m, int m_max, int64_t n, const void* res, void* out, int dtype,
                     int* status, cudaStream_t st);

// Launch `kernel` on `stream` as a programmatic dependent of the previous
// kernel in the stream (see grid_dep_wait).
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace fd_host
