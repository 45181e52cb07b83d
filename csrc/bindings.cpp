// Python bindings of the bitscom_b200 native extension (module bitscom_b200._C).
//
// Exposes:
//   * the standalone quantisation ops (reference-compatible layout and
//     semantics; reference bindings: cpp/src/lowbit_cuda_bindings.cpp:25-56),
//     all launched on the caller's current CUDA stream and free of host syncs;
//   * LowBitComm, the fused low-bit collective runtime;
//   * the `lowbit` c10d backend (registered from backend/process_group_lowbit.cpp).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <execinfo.h>
#include <unistd.h>

#include <csignal>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "backend/process_group_lowbit.h"
#include "kernels/launchers.h"
#include "runtime/comm.h"

namespace bitscom_b200 {
namespace {

// Debug aid: on SIGSEGV/SIGABRT print the native call stack (glibc
// backtrace) to stderr, then re-raise with the default action.
void crash_handler(int sig) {
  void* frames[64];
  const int n = backtrace(frames, 64);
  const char msg[] = "\n[bitscom] native backtrace:\n";
  (void)!write(2, msg, sizeof(msg) - 1);
  backtrace_symbols_fd(frames, n, 2);
  signal(sig, SIG_DFL);
  raise(sig);
}

void install_crash_backtrace() {
  signal(SIGSEGV, crash_handler);
  signal(SIGABRT, crash_handler);
}

DType to_dt(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return kF32;
    case at::kBFloat16: return kBF16;
    case at::kHalf: return kF16;
    default: TORCH_CHECK(false, "bitscom: expected a float32, bfloat16 or float16 tensor, got ", t);
  }
}

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "bitscom: ", name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), "bitscom: ", name, " must be contiguous");
}

cudaStream_t cur_stream(const at::Tensor& t) { return at::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

at::Tensor absmax_op(const at::Tensor& x, const c10::optional<at::Tensor>& residual) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto amax = at::zeros({1}, x.options().dtype(at::kInt));
  const auto s = cur_stream(x);
  if (residual && residual->defined()) {
    check_cuda(*residual, "residual");
    TORCH_CHECK(residual->scalar_type() == at::kFloat && residual->numel() == x.numel(), "bitscom: residual must be fp32 of x.numel()");
    launch::absmax_sum(x.data_ptr(), to_dt(x.scalar_type()), residual->data_ptr<float>(), x.numel(),
                       reinterpret_cast<uint32_t*>(amax.data_ptr<int>()), s);
  } else {
    launch::absmax(x.data_ptr(), to_dt(x.scalar_type()), x.numel(), reinterpret_cast<uint32_t*>(amax.data_ptr<int>()), s);
  }
  return amax.view(at::kFloat);
}

// Returns (packed | None, q16 | None, scale float64[1], amax float32[1]).
py::tuple quantize_op(const at::Tensor& x_in, int64_t bits, bool stochastic, int64_t seed, int64_t offset,
                      bool want_packed, bool want_q) {
  check_cuda(x_in, "x");
  auto x = x_in.contiguous();
  c10::cuda::CUDAGuard g(x.device());
  const auto s = cur_stream(x);
  const int64_t n = x.numel();
  auto amax = at::zeros({1}, x.options().dtype(at::kInt));
  launch::absmax(x.data_ptr(), to_dt(x.scalar_type()), n, reinterpret_cast<uint32_t*>(amax.data_ptr<int>()), s);
  auto scale = at::empty({1}, x.options().dtype(at::kDouble));
  at::Tensor packed, q;
  if (want_packed) packed = at::empty({packed_bytes_ref(n, static_cast<int>(bits))}, x.options().dtype(at::kByte));
  if (want_q) q = at::empty(x.sizes(), x.options().dtype(at::kShort));
  if (n == 0) {
    scale.fill_(1.0);
  } else {
    launch::quantize_ref(x.data_ptr(), to_dt(x.scalar_type()), n, static_cast<int>(bits),
                         reinterpret_cast<const uint32_t*>(amax.data_ptr<int>()), stochastic,
                         static_cast<uint64_t>(seed), static_cast<uint64_t>(offset),
                         want_packed ? packed.data_ptr<uint8_t>() : nullptr,
                         want_q ? q.data_ptr<int16_t>() : nullptr, scale.data_ptr<double>(), s);
  }
  py::object po = want_packed ? py::cast(packed) : py::none();
  py::object qo = want_q ? py::cast(q) : py::none();
  return py::make_tuple(po, qo, scale, amax.view(at::kFloat));
}

at::Tensor pack_op(const at::Tensor& q_in, int64_t bits) {
  check_cuda(q_in, "q");
  TORCH_CHECK(q_in.scalar_type() == at::kShort, "bitscom: pack expects int16 codes");
  auto q = q_in.contiguous();
  c10::cuda::CUDAGuard g(q.device());
  const int64_t n = q.numel();
  auto packed = at::empty({packed_bytes_ref(n, static_cast<int>(bits))}, q.options().dtype(at::kByte));
  launch::pack_ref(q.data_ptr<int16_t>(), n, static_cast<int>(bits), packed.data_ptr<uint8_t>(), cur_stream(q));
  return packed;
}

// Returns (q16 | None, out | None).
py::tuple unpack_op(const at::Tensor& packed_in, int64_t bits, int64_t numel, bool want_q,
                    c10::optional<at::ScalarType> out_dtype, double scale,
                    const c10::optional<at::Tensor>& scale_t) {
  check_cuda(packed_in, "packed");
  TORCH_CHECK(packed_in.scalar_type() == at::kByte, "bitscom: unpack expects uint8 bytes");
  auto packed = packed_in.contiguous();
  TORCH_CHECK(packed.numel() >= packed_bytes_ref(numel, static_cast<int>(bits)),
              "bitscom: packed buffer too small for ", numel, " codes of ", bits, " bits");
  c10::cuda::CUDAGuard g(packed.device());
  at::Tensor q, out, sc;
  if (want_q) q = at::empty({numel}, packed.options().dtype(at::kShort));
  if (out_dtype) out = at::empty({numel}, packed.options().dtype(*out_dtype));
  const float* sp = nullptr;
  if (scale_t && scale_t->defined()) {
    sc = scale_t->to(packed.device(), at::kFloat).contiguous();
    sp = sc.data_ptr<float>();
  }
  launch::unpack_ref(packed.data_ptr<uint8_t>(), numel, static_cast<int>(bits), want_q ? q.data_ptr<int16_t>() : nullptr,
                     out_dtype ? out.data_ptr() : nullptr, out_dtype ? to_dt(*out_dtype) : kF32,
                     static_cast<float>(scale), sp, cur_stream(packed));
  py::object qo = want_q ? py::cast(q) : py::none();
  py::object oo = out_dtype ? py::cast(out) : py::none();
  return py::make_tuple(qo, oo);
}

at::Tensor dequantize_op(const at::Tensor& q_in, double scale, const c10::optional<at::Tensor>& scale_t,
                         at::ScalarType out_dtype) {
  check_cuda(q_in, "q");
  TORCH_CHECK(q_in.scalar_type() == at::kShort, "bitscom: dequantize expects int16 codes");
  auto q = q_in.contiguous();
  c10::cuda::CUDAGuard g(q.device());
  auto out = at::empty(q.sizes(), q.options().dtype(out_dtype));
  at::Tensor sc;
  const float* sp = nullptr;
  if (scale_t && scale_t->defined()) {
    sc = scale_t->to(q.device(), at::kFloat).contiguous();
    sp = sc.data_ptr<float>();
  }
  launch::dequantize_i16(q.data_ptr<int16_t>(), q.numel(), out.data_ptr(), to_dt(out_dtype), static_cast<float>(scale), sp,
                         cur_stream(q));
  return out;
}

at::Tensor ef_roundtrip_op(const at::Tensor& x_in, const c10::optional<at::Tensor>& residual, int64_t bits,
                           bool stochastic, int64_t seed, int64_t offset) {
  check_cuda(x_in, "x");
  auto x = x_in.contiguous();
  c10::cuda::CUDAGuard g(x.device());
  const auto s = cur_stream(x);
  float* rp = nullptr;
  if (residual && residual->defined()) {
    check_cuda(*residual, "residual");
    TORCH_CHECK(residual->scalar_type() == at::kFloat && residual->numel() == x.numel(), "bitscom: residual must be fp32 of x.numel()");
    rp = residual->data_ptr<float>();
  }
  auto amax = at::zeros({1}, x.options().dtype(at::kInt));
  if (rp)
    launch::absmax_sum(x.data_ptr(), to_dt(x.scalar_type()), rp, x.numel(), reinterpret_cast<uint32_t*>(amax.data_ptr<int>()), s);
  else
    launch::absmax(x.data_ptr(), to_dt(x.scalar_type()), x.numel(), reinterpret_cast<uint32_t*>(amax.data_ptr<int>()), s);
  auto y = at::empty_like(x);
  launch::ef_roundtrip_ref(x.data_ptr(), to_dt(x.scalar_type()), x.numel(), static_cast<int>(bits), rp,
                           reinterpret_cast<const uint32_t*>(amax.data_ptr<int>()), stochastic,
                           static_cast<uint64_t>(seed), static_cast<uint64_t>(offset), y.data_ptr(), s);
  return y;
}

// ---------------------------------------------------------------------------
// LowBitComm bindings
// ---------------------------------------------------------------------------
ResidualBuf residual_ptr(const c10::optional<at::Tensor>& r, int64_t n, const at::Tensor& like) {
  if (!r || !r->defined()) return {};
  TORCH_CHECK(r->is_cuda() && r->is_contiguous() &&
                  (r->scalar_type() == at::kFloat || r->scalar_type() == at::kBFloat16),
              "bitscom: residual must be a contiguous fp32 or bf16 CUDA tensor");
  TORCH_CHECK(r->numel() == n, "bitscom: residual has ", r->numel(), " elements, expected ", n);
  TORCH_CHECK(r->device() == like.device(), "bitscom: residual is on another device");
  return ResidualBuf(r->data_ptr(), r->scalar_type() == at::kFloat ? kF32 : kBF16);
}

void comm_allreduce(LowBitComm& c, at::Tensor& t, const c10::optional<at::Tensor>& out_opt,
                    const c10::optional<at::Tensor>& residual, int64_t bits, int64_t fmt, int64_t algo,
                    bool sr, bool sr2, int64_t seed, int64_t offset, double post_scale, int64_t max_ctas) {
  check_cuda(t, "tensor");
  TORCH_CHECK(t.device().index() == c.device(), "bitscom: tensor is on cuda:", t.device().index(),
              " but the communicator lives on cuda:", c.device());
  at::Tensor out = out_opt && out_opt->defined() ? *out_opt : t;
  check_cuda(out, "out");
  TORCH_CHECK(out.numel() == t.numel() && out.scalar_type() == t.scalar_type(), "bitscom: out must match the input");
  c10::cuda::CUDAGuard g(t.device());
  c.allreduce(t.data_ptr(), out.data_ptr(), residual_ptr(residual, t.numel(), t), t.numel(), to_dt(t.scalar_type()),
              static_cast<int>(bits), static_cast<int>(fmt), static_cast<int>(algo), sr, sr2,
              static_cast<uint64_t>(seed), static_cast<uint64_t>(offset), static_cast<float>(post_scale),
              cur_stream(t), static_cast<int>(max_ctas));
}

void comm_reduce_scatter(LowBitComm& c, const at::Tensor& in, at::Tensor& out, const c10::optional<at::Tensor>& residual,
                         int64_t bits, int64_t fmt, bool sr, int64_t seed, int64_t offset, double post_scale,
                         int64_t max_ctas) {
  check_cuda(in, "input");
  check_cuda(out, "output");
  TORCH_CHECK(in.numel() == out.numel() * c.world(), "bitscom: reduce_scatter input must hold world * output elements");
  TORCH_CHECK(in.scalar_type() == out.scalar_type(), "bitscom: dtype mismatch");
  c10::cuda::CUDAGuard g(in.device());
  c.reduce_scatter(in.data_ptr(), out.data_ptr(), residual_ptr(residual, in.numel(), in), out.numel(),
                   to_dt(in.scalar_type()), static_cast<int>(bits), static_cast<int>(fmt), sr,
                   static_cast<uint64_t>(seed), static_cast<uint64_t>(offset), static_cast<float>(post_scale),
                   cur_stream(in), static_cast<int>(max_ctas));
}

void comm_all_gather(LowBitComm& c, const at::Tensor& in, at::Tensor& out, const c10::optional<at::Tensor>& residual,
                     int64_t bits, int64_t fmt, bool sr, int64_t seed, int64_t offset, int64_t max_ctas) {
  check_cuda(in, "input");
  check_cuda(out, "output");
  TORCH_CHECK(out.numel() == in.numel() * c.world(), "bitscom: all_gather output must hold world * input elements");
  TORCH_CHECK(in.scalar_type() == out.scalar_type(), "bitscom: dtype mismatch");
  c10::cuda::CUDAGuard g(in.device());
  c.all_gather(in.data_ptr(), out.data_ptr(), residual_ptr(residual, in.numel(), in), in.numel(),
               to_dt(in.scalar_type()), static_cast<int>(bits), static_cast<int>(fmt), sr,
               static_cast<uint64_t>(seed), static_cast<uint64_t>(offset), cur_stream(in),
               static_cast<int>(max_ctas));
}

}  // namespace
}  // namespace bitscom_b200

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using namespace bitscom_b200;
  m.doc() = "bitscom_b200 native extension: sm_100a low-bit kernels, fused NVLink collectives, lowbit c10d backend";
  m.def("absmax", &absmax_op, py::arg("x"), py::arg("residual") = py::none());
  m.def("quantize", &quantize_op, py::arg("x"), py::arg("bits"), py::arg("stochastic") = false,
        py::arg("seed") = 0, py::arg("offset") = 0, py::arg("want_packed") = true, py::arg("want_q") = false);
  m.def("pack", &pack_op, py::arg("q"), py::arg("bits"));
  m.def("unpack", &unpack_op, py::arg("packed"), py::arg("bits"), py::arg("numel"), py::arg("want_q") = true,
        py::arg("out_dtype") = py::none(), py::arg("scale") = 1.0, py::arg("scale_tensor") = py::none());
  m.def("dequantize", &dequantize_op, py::arg("q"), py::arg("scale") = 1.0, py::arg("scale_tensor") = py::none(),
        py::arg("out_dtype") = at::kFloat);
  m.def("ef_roundtrip", &ef_roundtrip_op, py::arg("x"), py::arg("residual") = py::none(), py::arg("bits") = 4,
        py::arg("stochastic") = false, py::arg("seed") = 0, py::arg("offset") = 0);
  m.def("install_crash_backtrace", &install_crash_backtrace,
        "print the native stack on SIGSEGV/SIGABRT (debugging aid)");
  m.def("packed_bytes", [](int64_t n, int64_t bits) -> int64_t { return packed_bytes_ref(n, static_cast<int>(bits)); });
  m.def("wire_sub_bytes", [](int64_t bits) -> int64_t { return launch::coll_sub_bytes(static_cast<int>(bits)); });
  m.def(
      "coll_schedule",
      [](int op, int world, int64_t items_per_slot, int64_t lag) {
        int a1, a2, a3;
        coll_phase_items(op, world, &a1, &a2, &a3);
        const int64_t total = (a1 + a2 + a3) * items_per_slot;
        std::vector<int64_t> order(static_cast<size_t>(total));
        for (int64_t t = 0; t < total; ++t) order[t] = coll_schedule_item(op, world, items_per_slot, lag, t);
        return order;
      },
      "Work item handed out for each ticket of a fused collective (the kernel's schedule, run on the host).",
      py::arg("op"), py::arg("world"), py::arg("items_per_slot"), py::arg("lag"));

  py::class_<CollStats>(m, "CollStats")
      .def_readonly("calls", &CollStats::calls)
      .def_readonly("launches", &CollStats::launches)
      .def_readonly("elements", &CollStats::elements)
      .def_readonly("wire_bytes", &CollStats::wire_bytes)
      .def_readonly("oneshot", &CollStats::oneshot)
      .def_readonly("twoshot", &CollStats::twoshot)
      .def_readonly("timed_launches", &CollStats::timed_launches)
      .def_readonly("kernel_ms", &CollStats::kernel_ms);

  py::class_<LowBitComm, std::shared_ptr<LowBitComm>>(m, "LowBitComm")
      .def(py::init<int, int, int, int64_t>(), py::arg("rank"), py::arg("world"), py::arg("device"),
           py::arg("workspace_bytes"))
      .def_property_readonly("rank", &LowBitComm::rank)
      .def_property_readonly("world", &LowBitComm::world)
      .def_property_readonly("device", &LowBitComm::device)
      .def_property_readonly("workspace_bytes", &LowBitComm::workspace_bytes)
      .def_property_readonly("ready", &LowBitComm::ready)
      .def_property_readonly("broken", &LowBitComm::broken)
      .def_property_readonly("epoch", &LowBitComm::epoch)
      .def("ipc_handle", [](const LowBitComm& c) {
        auto h = c.ipc_handle();
        return py::bytes(reinterpret_cast<const char*>(h.data()), h.size());
      })
      .def("open_peers", [](LowBitComm& c, const std::vector<py::bytes>& hs) {
        std::vector<std::vector<uint8_t>> v;
        for (const auto& b : hs) {
          std::string s = b;
          v.emplace_back(s.begin(), s.end());
        }
        c.open_peers(v);
      })
      .def("allreduce", &comm_allreduce, py::arg("tensor"), py::arg("out") = py::none(), py::arg("residual") = py::none(),
           py::arg("bits") = 4, py::arg("fmt") = 0, py::arg("algo") = 0, py::arg("stochastic") = false,
           py::arg("stochastic_requant") = false, py::arg("seed") = 0, py::arg("offset") = 0,
           py::arg("post_scale") = 1.0, py::arg("max_ctas") = 0)
      .def("reduce_scatter", &comm_reduce_scatter, py::arg("input"), py::arg("output"), py::arg("residual") = py::none(),
           py::arg("bits") = 8, py::arg("fmt") = 0, py::arg("stochastic") = false, py::arg("seed") = 0,
           py::arg("offset") = 0, py::arg("post_scale") = 1.0, py::arg("max_ctas") = 0)
      .def("all_gather", &comm_all_gather, py::arg("input"), py::arg("output"), py::arg("residual") = py::none(),
           py::arg("bits") = 8, py::arg("fmt") = 0, py::arg("stochastic") = false, py::arg("seed") = 0,
           py::arg("offset") = 0, py::arg("max_ctas") = 0)
      .def("status", &LowBitComm::status)
      .def("check", &LowBitComm::check)
      .def("set_timeout_ms", &LowBitComm::set_timeout_ms)
      .def("set_schedule_lag", &LowBitComm::set_schedule_lag)
      .def("device_epoch", &LowBitComm::device_epoch)
      .def("set_sub_per_item", &LowBitComm::set_sub_per_item)
      .def("set_kernel_variant", &LowBitComm::set_kernel_variant)
      .def_property_readonly("kernel_variant", &LowBitComm::kernel_variant)
      .def("set_ws_smem_budget", &LowBitComm::set_ws_smem_budget)
      .def("set_oneshot_max_bytes", &LowBitComm::set_oneshot_max_bytes)
      .def("set_tuning", &LowBitComm::set_tuning, py::arg("bits"), py::arg("fmt"), py::arg("oneshot_max_bytes"), py::arg("ws_min_bytes"))
      .def("oneshot_max_bytes", &LowBitComm::oneshot_max_bytes)
      .def("check_canaries", &LowBitComm::check_canaries)
      .def("sub_per_item", &LowBitComm::sub_per_item)
      .def("schedule_lag", &LowBitComm::schedule_lag)
      .def_property_readonly("timeout_ms", &LowBitComm::timeout_ms)
      .def("set_fault_skip_signal", &LowBitComm::set_fault_skip_signal)
      .def("max_elems_per_launch", &LowBitComm::max_elems_per_launch)
      .def("stats", &LowBitComm::stats)
      .def("set_timing", &LowBitComm::set_timing)
      .def_property_readonly("timing", &LowBitComm::timing)
      .def("reset_stats", &LowBitComm::reset_stats);

  register_backend_bindings(m);
}
