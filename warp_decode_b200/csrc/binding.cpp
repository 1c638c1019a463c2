// PyTorch extension surface of warp_decode_b200.
//
// Same function names, argument order and tensor contracts as the reference
// binding (csrc/binding.cpp:35-130 of Religious-J/warp_decode):
//   moe_gate_up_3d_batched(x[B,H] bf16, w[E,2I,H] bf16, topk_ids[B,K] int32) -> [B*K, I] bf16
//   moe_down_3d_batched(buffer[B*K,I] bf16, w[E,H,I] bf16, topk_ids[B,K] int32,
//                       topk_scale[B,K] fp32, B) -> [B, H] bf16
// Validation failures raise RuntimeError (TORCH_CHECK) before any launch,
// with the reference's messages for the checks the two share.  The output is
// allocated with the caching allocator and the kernels run on the current
// stream; nothing synchronises.  All compute goes through the C ABI in
// libwarp_decode_b200.so (include/warp_decode.h).
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "warp_decode.h"

namespace {

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be CUDA")
#define CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bf16")
#define CHECK_F32(x) TORCH_CHECK((x).scalar_type() == at::kFloat, #x " must be fp32")
#define CHECK_I32(x) TORCH_CHECK((x).scalar_type() == at::kInt, #x " must be int32")
#define CHECK_U8(x) TORCH_CHECK((x).scalar_type() == at::kByte, #x " must be uint8")

void check_same_device(const torch::Tensor& a, const torch::Tensor& b, const char* name) {
  TORCH_CHECK(a.device() == b.device(), name, " must be on the same device as the first input");
}

void check_rc(int rc) {
  TORCH_CHECK(rc == WD_OK, "warp_decode: ", wd_error_string(rc), ": ", wd_last_error_message());
}

int to_int(int64_t v, const char* what) {
  TORCH_CHECK(v >= 0 && v <= INT32_MAX, what, " out of int32 range");
  return static_cast<int>(v);
}

void* stream_ptr() { return reinterpret_cast<void*>(at::cuda::getCurrentCUDAStream().stream()); }

// Shared checks and shapes of the two gate_up entry points.
struct GateUpShape {
  int B, E, topk, hidden, inter;
};

GateUpShape gate_up_shape(const torch::Tensor& x, const torch::Tensor& w,
                          const torch::Tensor& topk_ids, bool mx) {
  CHECK_CUDA(x); CHECK_CONTIG(x); CHECK_BF16(x);
  CHECK_CUDA(w); CHECK_CONTIG(w);
  if (mx) { CHECK_U8(w); } else { CHECK_BF16(w); }
  CHECK_CUDA(topk_ids); CHECK_CONTIG(topk_ids); CHECK_I32(topk_ids);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 3 && topk_ids.dim() == 2);
  check_same_device(x, w, "w");
  check_same_device(x, topk_ids, "topk_ids");
  GateUpShape s;
  s.B = to_int(x.size(0), "B");
  s.hidden = to_int(x.size(1), "hidden");
  s.E = to_int(w.size(0), "E");
  const int two_i = to_int(w.size(1), "2*inter");
  TORCH_CHECK(two_i % 2 == 0, "w.size(1) must be 2 * inter");
  s.inter = two_i / 2;
  TORCH_CHECK(w.size(2) == s.hidden, "w.size(2) must == hidden");
  TORCH_CHECK(topk_ids.size(0) == s.B);
  s.topk = to_int(topk_ids.size(1), "topk");
  return s;
}

torch::Tensor moe_gate_up_3d_batched(torch::Tensor x, torch::Tensor w, torch::Tensor topk_ids) {
  const GateUpShape s = gate_up_shape(x, w, topk_ids, false);
  const c10::cuda::CUDAGuard guard(x.device());
  auto out = torch::empty({(int64_t)s.B * s.topk, s.inter}, x.options().dtype(at::kBFloat16));
  check_rc(wd_moe_gate_up_3d_batched(x.data_ptr(), w.data_ptr(), topk_ids.data_ptr<int32_t>(),
                                     out.data_ptr(), s.B, s.E, s.topk, s.hidden, s.inter, nullptr,
                                     stream_ptr()));
  return out;
}

torch::Tensor moe_gate_up_3d_batched_mxfp8(torch::Tensor x, torch::Tensor w_q,
                                           torch::Tensor w_scale, torch::Tensor topk_ids) {
  const GateUpShape s = gate_up_shape(x, w_q, topk_ids, true);
  CHECK_CUDA(w_scale); CHECK_CONTIG(w_scale); CHECK_U8(w_scale);
  check_same_device(x, w_scale, "w_scale");
  TORCH_CHECK(s.hidden % 32 == 0, "hidden must be a multiple of 32 for MXFP8 weights");
  TORCH_CHECK(w_scale.dim() == 3 && w_scale.size(0) == s.E && w_scale.size(1) == 2 * s.inter &&
                  w_scale.size(2) == s.hidden / 32,
              "w_scale must be [E, 2*inter, hidden/32]");
  const c10::cuda::CUDAGuard guard(x.device());
  auto out = torch::empty({(int64_t)s.B * s.topk, s.inter}, x.options().dtype(at::kBFloat16));
  check_rc(wd_moe_gate_up_3d_batched_mxfp8(
      x.data_ptr(), w_q.data_ptr<uint8_t>(), w_scale.data_ptr<uint8_t>(),
      topk_ids.data_ptr<int32_t>(), out.data_ptr(), s.B, s.E, s.topk, s.hidden, s.inter, nullptr,
      stream_ptr()));
  return out;
}

struct DownShape {
  int B, E, topk, hidden, inter;
};

DownShape down_shape(const torch::Tensor& buffer, const torch::Tensor& w,
                     const torch::Tensor& topk_ids, const torch::Tensor& topk_scale,
                     c10::optional<int64_t> B_arg, bool mx) {
  CHECK_CUDA(buffer); CHECK_CONTIG(buffer); CHECK_BF16(buffer);
  CHECK_CUDA(w); CHECK_CONTIG(w);
  if (mx) { CHECK_U8(w); } else { CHECK_BF16(w); }
  CHECK_CUDA(topk_ids); CHECK_CONTIG(topk_ids); CHECK_I32(topk_ids);
  CHECK_CUDA(topk_scale); CHECK_CONTIG(topk_scale); CHECK_F32(topk_scale);
  TORCH_CHECK(buffer.dim() == 2 && w.dim() == 3 && topk_ids.dim() == 2 && topk_scale.dim() == 2);
  check_same_device(buffer, w, "w");
  check_same_device(buffer, topk_ids, "topk_ids");
  check_same_device(buffer, topk_scale, "topk_scale");
  DownShape s;
  s.B = B_arg.has_value() ? to_int(*B_arg, "B") : to_int(topk_ids.size(0), "B");
  s.inter = to_int(buffer.size(1), "inter");
  s.E = to_int(w.size(0), "E");
  s.hidden = to_int(w.size(1), "hidden");
  TORCH_CHECK(w.size(2) == s.inter, "w.size(2) must == inter");
  TORCH_CHECK(topk_ids.size(0) == s.B);
  s.topk = to_int(topk_ids.size(1), "topk");
  TORCH_CHECK(topk_scale.size(0) == s.B && topk_scale.size(1) == s.topk);
  TORCH_CHECK(buffer.size(0) == (int64_t)s.B * s.topk, "buffer rows must be B*topk");
  return s;
}

torch::Tensor down_common(torch::Tensor buffer, torch::Tensor w, c10::optional<torch::Tensor> w_scale,
                          torch::Tensor topk_ids, torch::Tensor topk_scale,
                          c10::optional<int64_t> B_arg, bool fp32_out) {
  const bool mx = w_scale.has_value();
  const DownShape s = down_shape(buffer, w, topk_ids, topk_scale, B_arg, mx);
  if (mx) {
    const auto& sc = *w_scale;
    CHECK_CUDA(sc); CHECK_CONTIG(sc); CHECK_U8(sc);
    check_same_device(buffer, sc, "w_scale");
    TORCH_CHECK(s.inter % 32 == 0, "inter must be a multiple of 32 for MXFP8 weights");
    TORCH_CHECK(sc.dim() == 3 && sc.size(0) == s.E && sc.size(1) == s.hidden &&
                    sc.size(2) == s.inter / 32,
                "w_scale must be [E, hidden, inter/32]");
  }
  const c10::cuda::CUDAGuard guard(buffer.device());
  auto out = torch::empty({s.B, s.hidden},
                          buffer.options().dtype(fp32_out ? at::kFloat : at::kBFloat16));
  if (mx) {
    check_rc(wd_moe_down_3d_batched_mxfp8(
        buffer.data_ptr(), w.data_ptr<uint8_t>(), w_scale->data_ptr<uint8_t>(),
        topk_ids.data_ptr<int32_t>(), topk_scale.data_ptr<float>(), out.data_ptr(),
        fp32_out ? 1 : 0, s.B, s.E, s.topk, s.hidden, s.inter, nullptr, stream_ptr()));
  } else {
    check_rc(wd_moe_down_3d_batched(buffer.data_ptr(), w.data_ptr(), topk_ids.data_ptr<int32_t>(),
                                    topk_scale.data_ptr<float>(), out.data_ptr(), fp32_out ? 1 : 0,
                                    s.B, s.E, s.topk, s.hidden, s.inter, nullptr, stream_ptr()));
  }
  return out;
}

torch::Tensor moe_down_3d_batched(torch::Tensor buffer, torch::Tensor w, torch::Tensor topk_ids,
                                  torch::Tensor topk_scale, c10::optional<int64_t> B) {
  return down_common(buffer, w, c10::nullopt, topk_ids, topk_scale, B, false);
}

torch::Tensor moe_down_3d_batched_partial(torch::Tensor buffer, torch::Tensor w,
                                          torch::Tensor topk_ids, torch::Tensor topk_scale,
                                          c10::optional<int64_t> B) {
  return down_common(buffer, w, c10::nullopt, topk_ids, topk_scale, B, true);
}

torch::Tensor moe_down_3d_batched_mxfp8(torch::Tensor buffer, torch::Tensor w_q,
                                        torch::Tensor w_scale, torch::Tensor topk_ids,
                                        torch::Tensor topk_scale, c10::optional<int64_t> B,
                                        bool fp32_out) {
  return down_common(buffer, w_q, w_scale, topk_ids, topk_scale, B, fp32_out);
}

// gate_up -> down in one call (wd_moe_ffn_3d_batched; single launch for
// B*topk <= 64).  Uses the library's grid-barrier words of the device: calls
// on different streams of one device must not overlap.
torch::Tensor moe_ffn_3d_batched(torch::Tensor x, torch::Tensor w_gate_up, torch::Tensor w_down,
                                 torch::Tensor topk_ids, torch::Tensor topk_scale, bool fp32_out) {
  const GateUpShape s = gate_up_shape(x, w_gate_up, topk_ids, false);
  CHECK_CUDA(w_down); CHECK_CONTIG(w_down); CHECK_BF16(w_down);
  CHECK_CUDA(topk_scale); CHECK_CONTIG(topk_scale); CHECK_F32(topk_scale);
  check_same_device(x, w_down, "w_down");
  check_same_device(x, topk_scale, "topk_scale");
  TORCH_CHECK(w_down.dim() == 3 && w_down.size(0) == s.E && w_down.size(1) == s.hidden &&
                  w_down.size(2) == s.inter,
              "w_down must be [E, hidden, inter]");
  TORCH_CHECK(topk_scale.dim() == 2 && topk_scale.size(0) == s.B && topk_scale.size(1) == s.topk,
              "topk_scale must be [B, topk]");
  const c10::cuda::CUDAGuard guard(x.device());
  auto h = torch::empty({(int64_t)s.B * s.topk, s.inter}, x.options().dtype(at::kBFloat16));
  auto out = torch::empty({s.B, s.hidden}, x.options().dtype(fp32_out ? at::kFloat : at::kBFloat16));
  check_rc(wd_moe_ffn_3d_batched(x.data_ptr(), w_gate_up.data_ptr(), w_down.data_ptr(),
                                 topk_ids.data_ptr<int32_t>(), topk_scale.data_ptr<float>(),
                                 h.data_ptr(), nullptr, out.data_ptr(), fp32_out ? 1 : 0, s.B, s.E,
                                 s.topk, s.hidden, s.inter, nullptr, stream_ptr()));
  return out;
}

// Byte copies src[i] -> dst[i] (1-4 pairs of contiguous tensors of equal
// byte size) by the GPU's own loads and stores, one launch on the current
// stream of the pairs' CUDA device; host tensors must be pinned.
void copy_ranges(const std::vector<torch::Tensor>& src, const std::vector<torch::Tensor>& dst) {
  TORCH_CHECK(!src.empty() && src.size() == dst.size() && src.size() <= 4,
              "copy_ranges takes 1-4 (src, dst) pairs");
  c10::optional<at::Device> dev;
  const void* sp[4];
  void* dp[4];
  size_t nb[4];
  for (size_t i = 0; i < src.size(); ++i) {
    for (const torch::Tensor* t : {&src[i], &dst[i]}) {
      CHECK_CONTIG(*t);
      if (t->is_cuda()) {
        TORCH_CHECK(!dev || *dev == t->device(), "copy_ranges: CUDA tensors on more than one device");
        dev = t->device();
      } else {
        TORCH_CHECK(t->device().is_cpu() && (t->numel() == 0 || t->is_pinned()),
                    "copy_ranges: host tensors must be pinned");
      }
    }
    TORCH_CHECK(src[i].nbytes() == dst[i].nbytes(), "copy_ranges: src and dst sizes differ");
    sp[i] = src[i].data_ptr();
    dp[i] = dst[i].data_ptr();
    nb[i] = src[i].nbytes();
  }
  TORCH_CHECK(dev.has_value(), "copy_ranges: no CUDA tensor names the device");
  const c10::cuda::CUDAGuard guard(*dev);
  check_rc(wd_copy_ranges(sp, dp, nb, (int)src.size(), stream_ptr()));
}

// moe_ffn_3d_batched with x / topk_ids / topk_scale in pinned host memory and
// y returned in pinned host memory: inputs in (one copy launch), the FFN, y
// out (one copy launch), all on the current stream of the weights' device.
// (Storing y straight into the host buffer from the FFN's epilogues measured
// slower from 8 tokens up: 2-byte stores scattered over PCIe.)  Asynchronous
// like a non_blocking copy: read y after synchronising.
torch::Tensor moe_ffn_3d_batched_host(torch::Tensor x, torch::Tensor w_gate_up, torch::Tensor w_down,
                                      torch::Tensor topk_ids, torch::Tensor topk_scale,
                                      c10::optional<torch::Tensor> out, bool fp32_out) {
  for (const torch::Tensor* t : {&x, &topk_ids, &topk_scale}) {
    TORCH_CHECK(t->device().is_cpu() && (t->numel() == 0 || t->is_pinned()),
                "x, topk_ids and topk_scale must be pinned host tensors");
    CHECK_CONTIG(*t);
  }
  CHECK_BF16(x); CHECK_I32(topk_ids); CHECK_F32(topk_scale);
  CHECK_CUDA(w_gate_up);
  TORCH_CHECK(x.dim() == 2 && topk_ids.dim() == 2 && topk_scale.dim() == 2 &&
                  topk_ids.size(0) == x.size(0) && topk_scale.sizes() == topk_ids.sizes(),
              "x must be [B, hidden], topk_ids and topk_scale [B, topk]");
  const c10::cuda::CUDAGuard guard(w_gate_up.device());
  const int64_t xb = x.nbytes(), ib = topk_ids.nbytes(), sb = topk_scale.nbytes();
  const int64_t io = (xb + 15) / 16 * 16, so = io + (ib + 15) / 16 * 16;
  auto buf = torch::empty({so + sb}, w_gate_up.options().dtype(at::kByte));
  auto xd = buf.narrow(0, 0, xb).view(at::kBFloat16).view(x.sizes());
  auto idd = buf.narrow(0, io, ib).view(at::kInt).view(topk_ids.sizes());
  auto scd = buf.narrow(0, so, sb).view(at::kFloat).view(topk_scale.sizes());
  {
    const void* sp[3] = {x.data_ptr(), topk_ids.data_ptr(), topk_scale.data_ptr()};
    void* dp[3] = {xd.data_ptr(), idd.data_ptr(), scd.data_ptr()};
    const size_t nb[3] = {(size_t)xb, (size_t)ib, (size_t)sb};
    check_rc(wd_copy_ranges(sp, dp, nb, 3, stream_ptr()));
  }
  const auto ydt = fp32_out ? at::kFloat : at::kBFloat16;
  torch::Tensor yh;
  if (out.has_value()) {
    yh = *out;
    TORCH_CHECK(yh.device().is_cpu() && (yh.numel() == 0 || yh.is_pinned()) && yh.is_contiguous() &&
                    yh.scalar_type() == ydt && yh.dim() == 2 && yh.size(0) == x.size(0) &&
                    yh.size(1) == x.size(1),
                "out must be a pinned contiguous host tensor [B, hidden] of the output dtype");
  } else {
    yh = torch::empty({x.size(0), x.size(1)}, x.options().dtype(ydt).pinned_memory(true));
  }
  auto y = moe_ffn_3d_batched(xd, w_gate_up, w_down, idd, scd, fp32_out);
  const void* sp[1] = {y.data_ptr()};
  void* dp[1] = {yh.data_ptr()};
  const size_t nb[1] = {(size_t)y.nbytes()};
  check_rc(wd_copy_ranges(sp, dp, nb, 1, stream_ptr()));
  return yh;
}

// Router producer: (topk_ids int32 [B, topk], topk_weights fp32 [B, topk]).
std::tuple<torch::Tensor, torch::Tensor> moe_router_topk(torch::Tensor logits, int64_t topk,
                                                         bool renormalize) {
  CHECK_CUDA(logits); CHECK_CONTIG(logits);
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 || logits.scalar_type() == at::kFloat,
              "logits must be bf16 or fp32");
  TORCH_CHECK(logits.dim() == 2, "logits must be [B, E]");
  const int B = to_int(logits.size(0), "B");
  const int E = to_int(logits.size(1), "E");
  const int K = to_int(topk, "topk");
  const c10::cuda::CUDAGuard guard(logits.device());
  auto ids = torch::empty({B, K}, logits.options().dtype(at::kInt));
  auto w = torch::empty({B, K}, logits.options().dtype(at::kFloat));
  check_rc(wd_moe_router_topk(logits.data_ptr(), logits.scalar_type() == at::kFloat ? 1 : 0,
                              ids.data_ptr<int32_t>(), w.data_ptr<float>(), B, E, K,
                              renormalize ? 1 : 0, stream_ptr()));
  return {ids, w};
}

int64_t status(bool clear, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  uint32_t v = 0;
  check_rc(wd_status_read(&v, clear ? 1 : 0));
  return static_cast<int64_t>(v);
}

int64_t launch_count() { return static_cast<int64_t>(wd_launch_count()); }

void set_gate_up_path(int64_t path) { check_rc(wd_set_gate_up_path(static_cast<int>(path))); }
void set_down_path(int64_t path) { check_rc(wd_set_down_path(static_cast<int>(path))); }
void set_ffn_path(int64_t path) { check_rc(wd_set_ffn_path(static_cast<int>(path))); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  namespace py = pybind11;
  m.def("moe_gate_up_3d_batched", &moe_gate_up_3d_batched,
        "Fused MoE gate_up + silu_and_mul (bf16, FP32 accumulation)", py::arg("x"), py::arg("w"),
        py::arg("topk_ids"));
  m.def("moe_down_3d_batched", &moe_down_3d_batched,
        "Fused MoE down projection + top-k weighted sum (bf16 out)", py::arg("buffer"),
        py::arg("w"), py::arg("topk_ids"), py::arg("topk_scale"), py::arg("B") = py::none());
  m.def("moe_down_3d_batched_partial", &moe_down_3d_batched_partial,
        "As moe_down_3d_batched, FP32 output (tensor-parallel partial sums)", py::arg("buffer"),
        py::arg("w"), py::arg("topk_ids"), py::arg("topk_scale"), py::arg("B") = py::none());
  m.def("moe_gate_up_3d_batched_mxfp8", &moe_gate_up_3d_batched_mxfp8,
        "Fused MoE gate_up + silu_and_mul with MXFP8 (e4m3 + ue8m0/32) weights", py::arg("x"),
        py::arg("w_q"), py::arg("w_scale"), py::arg("topk_ids"));
  m.def("moe_down_3d_batched_mxfp8", &moe_down_3d_batched_mxfp8,
        "Fused MoE down + top-k weighted sum with MXFP8 weights", py::arg("buffer"),
        py::arg("w_q"), py::arg("w_scale"), py::arg("topk_ids"), py::arg("topk_scale"),
        py::arg("B") = py::none(), py::arg("fp32_out") = false);
  m.def("moe_ffn_3d_batched", &moe_ffn_3d_batched,
        "gate_up + silu*up + down + top-k weighted sum in one call (one launch for B*topk <= 64)",
        py::arg("x"), py::arg("w_gate_up"), py::arg("w_down"), py::arg("topk_ids"),
        py::arg("topk_scale"), py::arg("fp32_out") = false);
  m.def("copy_ranges", &copy_ranges,
        "byte copies src[i] -> dst[i] (1-4 pairs; device or pinned host tensors) in one launch",
        py::arg("src"), py::arg("dst"));
  m.def("moe_ffn_3d_batched_host", &moe_ffn_3d_batched_host,
        "moe_ffn_3d_batched on pinned host x / topk_ids / topk_scale, y returned in pinned host memory",
        py::arg("x"), py::arg("w_gate_up"), py::arg("w_down"), py::arg("topk_ids"),
        py::arg("topk_scale"), py::arg("out") = py::none(), py::arg("fp32_out") = false);
  m.def("moe_router_topk", &moe_router_topk,
        "top-k experts and routing weights from router logits [B, E] (bf16/fp32)",
        py::arg("logits"), py::arg("topk"), py::arg("renormalize") = true);
  m.def("status", &status, "Read (and clear) the device status word of the library",
        py::arg("clear") = true, py::arg("device") = 0);
  m.def("launch_count", &launch_count,
        "Kernels this library has enqueued in this process (graph captures count what they record)");
  m.def("set_gate_up_path", &set_gate_up_path,
        "gate_up kernel for later calls: 0 automatic, 1 SIMT, 2 tcgen05 tensor cores",
        py::arg("path"));
  m.def("set_down_path", &set_down_path,
        "down kernel for later calls: 0 automatic, 1 SIMT, 2 tcgen05 tensor cores",
        py::arg("path"));
  m.def("set_ffn_path", &set_ffn_path,
        "moe_ffn_3d_batched kernels for later calls: 0 automatic, 1 two launches, 2 one SIMT "
        "launch, 3 one tensor-core launch",
        py::arg("path"));
}
