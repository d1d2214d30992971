// Compiled dispatch of the operators' common case: tensors in, one C-ABI call,
// tensors out, with no Python between the caller and the launch.
//
// The Python operators (ops.py) check their arguments, describe each tensor
// as a row grid and pack a ctypes call: about 20 us of host time per call,
// several times a decode kernel's device time.  Each function here accepts
// the same arguments as its Python operator and, when every argument is on
// the common path (CUDA tensors of supported dtypes and matching shapes, at
// most four dimensions, no negative strides, out= that needs no copy), fills
// the same fd_rows / stride arguments the Python launcher would and calls the
// same entry point of libfd_b200.so on the tensor's device and current
// stream.  Anything else -- including every argument error -- returns None
// and the caller runs the Python path, which raises the reference's
// exception types and messages.  Both paths hand identical arguments to the
// kernels, so their results are bit-identical.
//
// The split-K workspaces (one zero-filled buffer per device and stream) live
// here and serve both paths.
#include <ATen/core/Tensor.h>
#include <ATen/ops/empty.h>
#include <ATen/ops/linear.h>
#include <ATen/ops/zeros.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <ATen/PythonTorchFunctionTLS.h>
#include <torch/csrc/autograd/python_variable.h>
#include <torch/csrc/utils/pybind.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "fd_b200.h"

namespace py = pybind11;

namespace {

constexpr int64_t kMaxM = 16;  // GEMV batch rows (kernels.GEMV_MAX_M)

// ------------------------------------------------------------ argument probes
// torch.Tensor and torch.nn.Parameter (which disables __torch_function__),
// looked up when the module is imported.
PyTypeObject* g_tensor_type = nullptr;
PyTypeObject* g_parameter_type = nullptr;

// A borrowed at::Tensor from a Python object, or nullptr when it is not one
// or must go through Python: any other Tensor subclass (it may override
// __torch_function__), any tensor while a torch-function mode is active
// (e.g. `with torch.device(...)`), or a tensor without storage.
const at::Tensor* as_tensor(py::handle h) {
  const PyTypeObject* type = Py_TYPE(h.ptr());
  if (type != g_tensor_type && type != g_parameter_type) return nullptr;
  if (at::impl::torch_function_mode_enabled()) return nullptr;
  const at::Tensor& t = THPVariable_Unpack(h.ptr());
  return t.has_storage() ? &t : nullptr;
}

bool as_float(py::handle h, double* v) {
  if (!PyFloat_Check(h.ptr()) && !PyLong_Check(h.ptr())) return false;
  *v = PyFloat_AsDouble(h.ptr());
  if (PyErr_Occurred()) {
    PyErr_Clear();
    return false;
  }
  return true;
}

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kHalf: return FD_F16;
    case at::kBFloat16: return FD_BF16;
    case at::kFloat: return FD_F32;
    default: return -1;
  }
}

bool activation(const at::Tensor& t) {
  return t.is_cuda() && (t.scalar_type() == at::kHalf || t.scalar_type() == at::kBFloat16);
}

bool same_meta(const at::Tensor& t, const at::Tensor& like) {
  return t.sizes() == like.sizes() && t.scalar_type() == like.scalar_type() && t.device() == like.device();
}

// ops.py's row grid (kernels.row_layout) without the copies: at most four
// dimensions and no negative stride, else not on the fast path.
bool rows_of(const at::Tensor& t, fd_rows* r) {
  const int64_t nd = t.dim();
  if (nd < 1 || nd > 4) return false;
  for (int64_t d = 0; d < nd; ++d)
    if (t.stride(d) < 0) return false;
  int64_t sz[3] = {1, 1, 1}, st[3] = {0, 0, 0};
  const int64_t lead = nd - 1;
  for (int64_t d = 0; d < lead; ++d) {
    sz[3 - lead + d] = t.size(d);
    st[3 - lead + d] = t.stride(d);
  }
  std::memset(r, 0, sizeof(*r));
  r->ptr = t.data_ptr();
  r->dtype = dtype_code(t.scalar_type());
  r->a = sz[0]; r->b = sz[1]; r->c = sz[2];
  r->sa = st[0]; r->sb = st[1]; r->sc = st[2];
  r->col = t.stride(nd - 1);
  r->n = t.size(nd - 1);
  return true;
}

int64_t row_count(const fd_rows& r) { return r.a * r.b * r.c; }

void check(int status, const char* what) {
  if (status != FD_OK)
    throw std::runtime_error(std::string(what) + " failed: " + fd_status_string(status) + " (status " +
                             std::to_string(status) + ")");
}

void* stream_of(const at::Tensor& t) { return c10::cuda::getCurrentCUDAStream(t.get_device()).stream(); }

// kind=None reads $FUSED_DECODE_LINEAR_KIND (default "dot"), as
// kernels.resolve_kind does; an unknown kind is left to the Python path.
bool kind_of(py::handle h, int* kind) {
  std::string s;
  if (h.is_none()) {
    const char* env = std::getenv("FUSED_DECODE_LINEAR_KIND");
    s = env ? env : "dot";
  } else if (PyUnicode_Check(h.ptr())) {
    s = py::cast<std::string>(h);
  } else {
    return false;
  }
  if (s == "dot") *kind = FD_KIND_DOT;
  else if (s == "simt") *kind = FD_KIND_SIMT;
  else return false;
  return true;
}

// ------------------------------------------------------------ workspaces
struct WsKey {
  int dev;
  uintptr_t stream;
  bool operator<(const WsKey& o) const { return dev != o.dev ? dev < o.dev : stream < o.stream; }
};

std::mutex g_ws_mu;
// never destroyed: device buffers must not be freed by static destructors at exit
auto* g_ws = new std::map<WsKey, at::Tensor>();

at::Tensor workspace_for(int dev, size_t bytes) {
  const cudaStream_t st = c10::cuda::getCurrentCUDAStream(dev).stream();
  std::lock_guard<std::mutex> lock(g_ws_mu);
  at::Tensor& t = (*g_ws)[WsKey{dev, reinterpret_cast<uintptr_t>(st)}];
  if (!t.defined() || static_cast<size_t>(t.numel()) < bytes) {
    const int64_t size = static_cast<int64_t>(std::max<size_t>(bytes, size_t{1} << 20));
    t = at::zeros({size}, at::TensorOptions().dtype(at::kByte).device(at::kCUDA, dev));
  }
  return t;
}

// ------------------------------------------------------------ norms
bool norm_weight_ok(const at::Tensor& w, const at::Tensor& x) {
  return w.device() == x.device() && dtype_code(w.scalar_type()) >= 0 && w.dim() == 1 && x.dim() >= 1 &&
         w.size(0) == x.size(-1);
}

bool eps_ok(py::handle h, double* eps) { return as_float(h, eps) && std::isfinite(*eps) && *eps >= 0.0; }

// out= given: same shape, dtype and device as x, and a grid the kernels can
// address in place.  Not given: a fresh contiguous tensor.
bool out_for(py::handle h, const at::Tensor& like, at::Tensor* out, fd_rows* r) {
  if (h.is_none()) {
    *out = at::empty(like.sizes(), like.options());
  } else {
    const at::Tensor* o = as_tensor(h);
    if (!o || !same_meta(*o, like)) return false;
    *out = *o;
  }
  return rows_of(*out, r);
}

py::object rms_norm(py::handle hx, py::handle hw, py::handle heps, py::handle hout) {
  const at::Tensor* x = as_tensor(hx);
  const at::Tensor* w = as_tensor(hw);
  double eps;
  if (!x || !w || !activation(*x) || !norm_weight_ok(*w, *x) || !eps_ok(heps, &eps)) return py::none();
  fd_rows rx, ry;
  if (!rows_of(*x, &rx)) return py::none();
  const c10::cuda::CUDAGuard guard(x->device());
  at::Tensor out;
  if (!out_for(hout, *x, &out, &ry)) return py::none();
  if (row_count(rx) > 0 && rx.n > 0)
    check(fd_rms_out(&rx, nullptr, w->data_ptr(), dtype_code(w->scalar_type()), w->stride(0), &ry, nullptr,
                     static_cast<float>(eps), stream_of(*x)),
          "fd_rms_out");
  return py::cast(out);
}

py::object add_rms_norm(py::handle hx, py::handle hr, py::handle hw, py::handle heps, py::handle hout,
                        py::handle hres_out) {
  const at::Tensor* x = as_tensor(hx);
  const at::Tensor* r = as_tensor(hr);
  const at::Tensor* w = as_tensor(hw);
  double eps;
  if (!x || !r || !w || !activation(*x) || !activation(*r) || !same_meta(*r, *x) || !norm_weight_ok(*w, *x) ||
      !eps_ok(heps, &eps))
    return py::none();
  fd_rows rx, rr, ry, rro;
  if (!rows_of(*x, &rx) || !rows_of(*r, &rr)) return py::none();
  const c10::cuda::CUDAGuard guard(x->device());
  at::Tensor out, res_out;
  if (!out_for(hout, *x, &out, &ry) || !out_for(hres_out, *x, &res_out, &rro)) return py::none();
  if (row_count(rx) > 0 && rx.n > 0)
    check(fd_rms_out(&rx, &rr, w->data_ptr(), dtype_code(w->scalar_type()), w->stride(0), &ry, &rro,
                     static_cast<float>(eps), stream_of(*x)),
          "fd_rms_out");
  return py::make_tuple(out, res_out);
}

// ------------------------------------------------------------ rope, swiglu
py::object rope(py::handle hx, py::handle hc, py::handle hs, py::handle hout) {
  const at::Tensor* x = as_tensor(hx);
  const at::Tensor* c = as_tensor(hc);
  const at::Tensor* s = as_tensor(hs);
  if (!x || !c || !s || !activation(*x) || x->dim() < 1 || x->size(-1) % 2 != 0) return py::none();
  for (const at::Tensor* a : {c, s})
    if (a->device() != x->device() || dtype_code(a->scalar_type()) < 0 || a->dim() < 1 ||
        a->dim() > x->dim() || a->size(-1) != x->size(-1))
      return py::none();
  // right-aligned broadcast, as Tensor.expand: every angle dim is 1 or x's
  for (const at::Tensor* a : {c, s})
    for (int64_t d = 1; d <= a->dim(); ++d)
      if (a->size(-d) != 1 && a->size(-d) != x->size(-d)) return py::none();
  const at::Tensor cb = c->expand(x->sizes());
  const at::Tensor sb = s->expand(x->sizes());
  fd_rows rx, rc, rs, ry;
  if (!rows_of(*x, &rx) || !rows_of(cb, &rc) || !rows_of(sb, &rs)) return py::none();
  const c10::cuda::CUDAGuard guard(x->device());
  at::Tensor out;
  if (!out_for(hout, *x, &out, &ry)) return py::none();
  if (row_count(rx) > 0 && rx.n > 0) check(fd_rope_out(&rx, &rc, &rs, &ry, stream_of(*x)), "fd_rope_out");
  return py::cast(out);
}

py::object swiglu(py::handle hg, py::handle hu, py::handle hout) {
  const at::Tensor* g = as_tensor(hg);
  const at::Tensor* u = as_tensor(hu);
  if (!g || !u || !activation(*g) || !activation(*u) || !same_meta(*u, *g)) return py::none();
  fd_rows rg, ru, ry;
  if (!rows_of(*g, &rg) || !rows_of(*u, &ru)) return py::none();
  const c10::cuda::CUDAGuard guard(g->device());
  at::Tensor out;
  if (!out_for(hout, *g, &out, &ry)) return py::none();
  if (row_count(rg) > 0 && rg.n > 0) check(fd_swiglu_out(&rg, &ru, &ry, stream_of(*g)), "fd_swiglu_out");
  return py::cast(out);
}

// ------------------------------------------------------------ linear_decode
// ops.linear_decode's row_add forms that need no copy: a 1-D row of N, the
// full output shape contiguous, or a 2-D [1|M, 1|N] grid.
bool row_add_strides(const at::Tensor& ra, int64_t m, int64_t n, c10::IntArrayRef expected, int64_t* srm,
                     int64_t* srn) {
  if (ra.dim() == 1 && ra.numel() == n) {
    *srm = 0;
    *srn = n == 1 ? 0 : ra.stride(0);
    return true;
  }
  if (ra.sizes() == expected && ra.is_contiguous()) {
    *srm = m == 1 ? 0 : n;
    *srn = n == 1 ? 0 : 1;
    return true;
  }
  if (ra.dim() == 2 && (ra.size(0) == 1 || ra.size(0) == m) && (ra.size(1) == 1 || ra.size(1) == n)) {
    *srm = ra.size(0) == 1 ? 0 : ra.stride(0);
    *srn = ra.size(1) == 1 ? 0 : ra.stride(1);
    return true;
  }
  return false;
}

// x as [M, K] without a copy (ops._as_mk): 2-D with non-negative strides as
// it is, or contiguous of any rank viewed as [-1, K]; else not on the fast path.
bool as_mk(const at::Tensor& x, int64_t* m, int64_t* sxm, int64_t* sxk) {
  const int64_t k = x.size(-1);
  if (x.dim() == 2 && x.stride(0) >= 0 && x.stride(1) >= 0) {
    *m = x.size(0);
    *sxm = x.stride(0);
    *sxk = x.stride(1);
    return true;
  }
  if (!x.is_contiguous()) return false;
  *m = k == 0 ? 0 : x.numel() / k;
  *sxm = k;
  *sxk = 1;
  return true;
}

py::object linear_decode(py::handle hx, py::handle hw, py::handle hb, py::handle hra, py::handle hout,
                         py::handle hkind) {
  const at::Tensor* x = as_tensor(hx);
  const at::Tensor* w = as_tensor(hw);
  int kind;
  if (!x || !w || !activation(*x) || x->dim() < 1 || w->dim() != 2 || w->device() != x->device() ||
      w->scalar_type() != x->scalar_type() || !kind_of(hkind, &kind))
    return py::none();
  const int64_t n = w->size(0), k = w->size(1);
  if (x->size(-1) != k) return py::none();
  int64_t sxm, sxk, m;
  if (!as_mk(*x, &m, &sxm, &sxk)) return py::none();
  if (m < 1 || n < 1 || k < 1) return py::none();
  std::vector<int64_t> expected(x->sizes().begin(), x->sizes().end() - 1);
  expected.push_back(n);
  if (m > kMaxM) {
    // Wider batches pass through to F.linear, as ops.linear_decode does; only
    // the plain form (no row_add, no out=, bias absent or of x's dtype).
    if (!hra.is_none() || !hout.is_none()) return py::none();
    std::optional<at::Tensor> b;
    if (!hb.is_none()) {
      const at::Tensor* bt = as_tensor(hb);
      if (!bt || bt->dim() != 1 || bt->size(0) != n || bt->device() != x->device() ||
          bt->scalar_type() != x->scalar_type())
        return py::none();
      b = *bt;
    }
    const at::Tensor x2 = x->dim() == 2 ? *x : x->view({-1, k});
    return py::cast(at::linear(x2, *w, b).view(expected));
  }
  const void* bias = nullptr;
  int bias_dt = 0;
  int64_t sbias = 0;
  if (!py::handle(hb).is_none()) {
    const at::Tensor* b = as_tensor(hb);
    if (!b || b->dim() != 1 || b->size(0) != n || b->device() != x->device() ||
        (b->scalar_type() != x->scalar_type() && b->scalar_type() != at::kFloat))
      return py::none();
    bias = b->data_ptr();
    bias_dt = dtype_code(b->scalar_type());
    sbias = b->stride(0);
  }
  const void* ra_ptr = nullptr;
  int ra_dt = 0;
  int64_t srm = 0, srn = 0;
  if (!hra.is_none()) {
    const at::Tensor* ra = as_tensor(hra);
    if (!ra || ra->device() != x->device() || dtype_code(ra->scalar_type()) < 0 ||
        !row_add_strides(*ra, m, n, expected, &srm, &srn))
      return py::none();
    ra_ptr = ra->data_ptr();
    ra_dt = dtype_code(ra->scalar_type());
  }
  const c10::cuda::CUDAGuard guard(x->device());
  at::Tensor y;
  if (hout.is_none()) {
    y = at::empty(expected, x->options());
  } else {
    const at::Tensor* o = as_tensor(hout);
    if (!o || o->sizes() != c10::IntArrayRef(expected) || o->scalar_type() != x->scalar_type() ||
        o->device() != x->device() || !o->is_contiguous())
      return py::none();
    y = *o;
  }
  const size_t ws_bytes = fd_linear_workspace_bytes(static_cast<int32_t>(m), n, k);
  const at::Tensor ws = workspace_for(x->get_device(), ws_bytes);
  check(fd_linear_out(x->data_ptr(), sxm, sxk, w->data_ptr(), w->stride(0), w->stride(1), bias, bias_dt, sbias,
                      ra_ptr, ra_dt, srm, srn, y.data_ptr(), n, 1, dtype_code(x->scalar_type()),
                      static_cast<int32_t>(m), n, k, kind, ws.data_ptr(), static_cast<size_t>(ws.numel()),
                      stream_of(*x)),
        "fd_linear_out");
  return py::cast(y);
}

// ------------------------------------------------------------ post_attn_mlp
// kernels.mlp_fusable: the two fused kernels can address these operands.
bool mlp_fusable(const at::Tensor& hidden, const at::Tensor& nw, const at::Tensor& wgu, const at::Tensor& wd,
                 int64_t m, int64_t h, int64_t i) {
  if (m < 1 || m > kMaxM || h % 8 || i % 8 || i == 0) return false;
  if (!hidden.is_contiguous() || nw.stride(0) != 1) return false;
  if (wgu.stride(1) != 1 || wd.stride(1) != 1 || wgu.stride(0) % 8 || wd.stride(0) % 8) return false;
  for (const at::Tensor* t : {&hidden, &nw, &wgu, &wd})
    if (reinterpret_cast<uintptr_t>(t->data_ptr()) % 16) return false;
  // the gate/up kernel's smallest ring (2 stages) with the resident or the
  // streamed batch (kernels.mlp_fusable)
  const int64_t ks = (h + 127) / 128;
  const int64_t nes = nw.scalar_type() == at::kFloat ? 4 : 2;
  const int64_t fixed = 1024 + 2 * 32768 + 64 * 16 * 4 + 2 * 12 * 8;
  const int64_t resident = fixed + ks * 2 * m * 128 + ((h * nes + 15) & ~int64_t{15});
  const int64_t streamed = fixed + 2 * 2 * (m <= 8 ? 1024 : 2048);
  return std::min(resident, streamed) <= 227 * 1024 - 1024;
}

py::object post_attn_mlp(py::handle hh, py::handle hnw, py::handle hgu, py::handle hd, py::handle heps,
                         py::handle hkind) {
  const at::Tensor* hid = as_tensor(hh);
  const at::Tensor* nw = as_tensor(hnw);
  const at::Tensor* wgu = as_tensor(hgu);
  const at::Tensor* wd = as_tensor(hd);
  double eps;
  int kind;
  if (!hid || !nw || !wgu || !wd || !activation(*hid) || hid->dim() < 1 || wgu->dim() != 2 || wd->dim() != 2 ||
      !eps_ok(heps, &eps) || !kind_of(hkind, &kind))
    return py::none();
  const int64_t h = wgu->size(1), i = wd->size(1);
  if (wgu->size(0) != 2 * i || wd->size(0) != h || hid->size(-1) != h) return py::none();
  if (wgu->scalar_type() != hid->scalar_type() || wd->scalar_type() != hid->scalar_type()) return py::none();
  if (wgu->device() != hid->device() || wd->device() != hid->device() || !norm_weight_ok(*nw, *hid))
    return py::none();
  const int64_t m = h == 0 ? 0 : hid->numel() / h;
  if (!mlp_fusable(*hid, *nw, *wgu, *wd, m, h, i)) return py::none();
  const c10::cuda::CUDAGuard guard(hid->device());
  at::Tensor out = at::empty(hid->sizes(), hid->options());
  const size_t ws_bytes = fd_post_attn_mlp_workspace_bytes(static_cast<int32_t>(m), h, i);
  const at::Tensor ws = workspace_for(hid->get_device(), ws_bytes);
  const int dt = dtype_code(hid->scalar_type());
  check(fd_post_attn_mlp_out(hid->data_ptr(), nw->data_ptr(), dtype_code(nw->scalar_type()), wgu->data_ptr(),
                             wgu->stride(0), wd->data_ptr(), wd->stride(0), out.data_ptr(), dt, dt,
                             static_cast<int32_t>(m), h, i, static_cast<float>(eps), kind, 1, ws.data_ptr(),
                             static_cast<size_t>(ws.numel()), stream_of(*hid)),
        "fd_post_attn_mlp_out");
  return py::cast(out);
}

// ------------------------------------------------------------ test hooks
// The arguments the fast path derives from a tensor's layout, for any device,
// so tests can compare them with the Python path's without a GPU.
py::object layout_rows(py::handle h) {
  const at::Tensor* t = as_tensor(h);
  fd_rows r;
  if (!t || !rows_of(*t, &r)) return py::none();
  return py::make_tuple(r.a, r.b, r.c, r.sa, r.sb, r.sc, r.col, r.n);
}

// (m, sxm, sxk, srm, srn) for x [..., K] against an [n, K] weight and an
// optional row_add, or None where the fast path would decline.
py::object layout_linear(py::handle hx, int64_t n, py::handle hra) {
  const at::Tensor* x = as_tensor(hx);
  int64_t m, sxm, sxk, srm = 0, srn = 0;
  if (!x || x->dim() < 1 || !as_mk(*x, &m, &sxm, &sxk)) return py::none();
  if (!hra.is_none()) {
    std::vector<int64_t> expected(x->sizes().begin(), x->sizes().end() - 1);
    expected.push_back(n);
    const at::Tensor* ra = as_tensor(hra);
    if (!ra || !row_add_strides(*ra, m, n, expected, &srm, &srn)) return py::none();
  }
  return py::make_tuple(m, sxm, sxk, srm, srn);
}

// ------------------------------------------------------------ workspace API
at::Tensor workspace(int64_t device, int64_t nbytes) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  return workspace_for(static_cast<int>(device), static_cast<size_t>(std::max<int64_t>(nbytes, 0)));
}

py::list workspaces() {
  py::list out;
  std::lock_guard<std::mutex> lock(g_ws_mu);
  for (const auto& kv : *g_ws) out.append(py::make_tuple(py::make_tuple(kv.first.dev, kv.first.stream), kv.second));
  return out;
}

void clear_workspaces() {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  g_ws->clear();
}

}  // namespace

PYBIND11_MODULE(_fastpath, mod) {
  mod.doc() = "Compiled common-case dispatch of the fused_decode_b200 operators (None = use the Python path)";
  // module-lifetime references (never released: the types outlive the module)
  g_tensor_type = reinterpret_cast<PyTypeObject*>(py::object(py::module_::import("torch").attr("Tensor")).release().ptr());
  g_parameter_type =
      reinterpret_cast<PyTypeObject*>(py::object(py::module_::import("torch.nn").attr("Parameter")).release().ptr());
  mod.def("rms_norm", &rms_norm);
  mod.def("add_rms_norm", &add_rms_norm);
  mod.def("rope", &rope);
  mod.def("swiglu", &swiglu);
  mod.def("linear_decode", &linear_decode);
  mod.def("post_attn_mlp", &post_attn_mlp);
  mod.def("layout_rows", &layout_rows);
  mod.def("layout_linear", &layout_linear);
  mod.def("workspace", &workspace);
  mod.def("workspaces", &workspaces);
  mod.def("clear_workspaces", &clear_workspaces);
}
