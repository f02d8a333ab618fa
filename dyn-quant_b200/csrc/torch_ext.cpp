// torch_ext.cpp -- the dyn_quant._C torch extension: the reference's four
// bindings (csrc/bindings.cpp:184-193 of dyn-quant) with the same names,
// argument meaning and RuntimeError behaviour, implemented over the C ABI of
// libdq_b200.so.  Extra functions: build_colmajor, build_native, detect_outliers,
// split_gemv_batched.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "../../include/dq_abi.h"

namespace {

// GEMV workspace per (device, stream), zero-filled when allocated and grown on
// demand.  The kernels leave the parts that must start at zero (counters,
// published partial sums) at zero after every call, so it is reused as is;
// calls on one stream are ordered, and each stream has its own.  Kept for the
// life of the process (never destroyed: no CUDA calls during static
// destruction).
std::mutex& workspace_mu() {
    static std::mutex mu;
    return mu;
}
std::map<std::pair<int, void*>, torch::Tensor>& workspace_cache() {
    static auto* cache = new std::map<std::pair<int, void*>, torch::Tensor>();
    return *cache;
}

torch::Tensor workspace_for(const torch::Device& dev, void* stream, size_t bytes) {
    std::lock_guard<std::mutex> lock(workspace_mu());
    auto* cache = &workspace_cache();
    const auto key = std::make_pair(static_cast<int>(dev.index()), stream);
    auto it = cache->find(key);
    if (it == cache->end() || static_cast<size_t>(it->second.numel()) < bytes) {
        const int64_t n = static_cast<int64_t>((bytes + 4095) / 4096 * 4096);
        (*cache)[key] = torch::zeros({n}, torch::TensorOptions().dtype(torch::kUInt8).device(dev));
        it = cache->find(key);
    }
    return it->second;
}

// Zero-fill every cached workspace on its own stream (after
// dq_read_device_error reported an error; see include/dq_abi.h).
void reset_workspaces() {
    std::lock_guard<std::mutex> lock(workspace_mu());
    for (auto& kv : workspace_cache()) {
        const auto& t = kv.second;
        const at::cuda::CUDAGuard guard(t.device());
        const dq_status_t s = dq_reset_workspace(t.data_ptr(), static_cast<size_t>(t.numel()), kv.first.second);
        TORCH_CHECK(s == DQ_OK, "reset_workspaces failed: ", dq_status_string(s));
    }
}

void check_status(dq_status_t s, const char* what) {
    if (s == DQ_OK) return;
    if (s == DQ_ERR_CUDA)
        TORCH_CHECK(false, what, " failed: ", dq_status_string(s), " (cudaError ", dq_last_cuda_error(), ")");
    TORCH_CHECK(false, what, " failed: ", dq_status_string(s));
}

// csrc/bindings.cpp:14-18
void check_fp16_contiguous(const torch::Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
    TORCH_CHECK(t.scalar_type() == at::kHalf, name, " must be float16");
}

void* stream_of(const torch::Tensor&) { return at::cuda::getCurrentCUDAStream().stream(); }

const uint16_t* h16(const torch::Tensor& t) { return reinterpret_cast<const uint16_t*>(t.data_ptr()); }
uint16_t* h16m(torch::Tensor& t) { return reinterpret_cast<uint16_t*>(t.data_ptr()); }

// The FP16 weights may be the row-major [d_out, d_in] copy the reference keeps,
// or the transposed view of the column-major mirror (stride (1, d_out)) that
// DynQuantLinear keeps; both are [d_out, d_in] tensors with the same values.
struct Fp16View {
    const uint16_t* rm = nullptr;
    const uint16_t* cm = nullptr;
};

Fp16View fp16_view(const torch::Tensor& w) {
    TORCH_CHECK(w.dim() == 2, "fp16_weights must be 2D");
    TORCH_CHECK(w.is_cuda(), "fp16_weights must be a CUDA tensor");
    TORCH_CHECK(w.scalar_type() == at::kHalf, "fp16_weights must be float16");
    Fp16View v;
    if (w.is_contiguous()) {
        v.rm = h16(w);
    } else if (w.t().is_contiguous()) {
        v.cm = h16(w);
    } else {
        TORCH_CHECK(false, "fp16_weights must be contiguous (row-major) or the transpose of a contiguous column-major mirror");
    }
    return v;
}

// csrc/bindings.cpp:94-111 plus the shape checks the reference leaves implicit.
dq_weights_t make_weights(const torch::Tensor& packed, const torch::Tensor& scales,
                          const torch::Tensor& zeros, const torch::Tensor& fp16_w,
                          const torch::Tensor& x, bool need_fp16,
                          const c10::optional<torch::Tensor>& native) {
    TORCH_CHECK(fp16_w.dim() == 2, "fp16_weights must be 2D");
    check_fp16_contiguous(scales, "scales");
    check_fp16_contiguous(zeros, "zeros");
    check_fp16_contiguous(x, "x");
    TORCH_CHECK(packed.is_cuda() && packed.is_contiguous() && packed.scalar_type() == at::kByte,
                "packed must be a contiguous CUDA uint8 tensor");
    const int64_t d_out = fp16_w.size(0), d_in = fp16_w.size(1);
    TORCH_CHECK(d_in % 128 == 0, "d_in must be divisible by GROUP_SIZE=128");
    TORCH_CHECK(x.numel() == d_in, "x length must equal d_in=", d_in);
    TORCH_CHECK(packed.dim() == 2 && packed.size(0) == d_out && packed.size(1) == d_in / 2,
                "packed column mismatch");
    TORCH_CHECK(scales.numel() == d_out * (d_in / 128) && zeros.numel() == d_out * (d_in / 128),
                "scales/zeros must hold d_out * d_in/128 values");
    TORCH_CHECK(x.device() == packed.device() && x.device() == fp16_w.device() &&
                    x.device() == scales.device() && x.device() == zeros.device(),
                "all tensors must be on the same device");
    dq_weights_t w{};
    w.packed = reinterpret_cast<const uint8_t*>(packed.data_ptr());
    w.scales = h16(scales);
    w.zeros = h16(zeros);
    if (need_fp16) {
        Fp16View v = fp16_view(fp16_w);
        w.fp16 = v.rm;
        w.fp16_cm = v.cm;
    }
    if (native.has_value() && native->defined()) {
        const auto& nv = *native;
        TORCH_CHECK(nv.is_cuda() && nv.is_contiguous() && nv.device() == x.device(),
                    "native must be a contiguous CUDA tensor on x's device");
        TORCH_CHECK(static_cast<size_t>(nv.numel() * nv.element_size()) ==
                        dq_native_bytes(static_cast<int32_t>(d_out), static_cast<int32_t>(d_in)),
                    "native layout size does not match the weight shape");
        w.native = reinterpret_cast<const uint8_t*>(nv.data_ptr());
    }
    w.d_out = static_cast<int32_t>(d_out);
    w.d_in = static_cast<int32_t>(d_in);
    return w;
}

// quantize_weights(weight [d_out, d_in] f16) -> (packed, scales, zeros, fp16_copy)
// (csrc/bindings.cpp:25-75; quantized on the device, bit-exact with the host loop).
// with_copy=false returns an undefined (None) fp16_copy: for callers that keep
// the weights in another form (DynQuantLinear keeps the column-major mirror).
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor>
quantize_weights(const torch::Tensor& weight, bool with_copy) {
    check_fp16_contiguous(weight, "weight");
    TORCH_CHECK(weight.dim() == 2, "weight must be 2D [d_out, d_in]");
    const int64_t d_out = weight.size(0), d_in = weight.size(1);
    TORCH_CHECK(d_in % 128 == 0, "d_in must be divisible by GROUP_SIZE=", 128);
    const at::cuda::CUDAGuard guard(weight.device());
    auto u8 = torch::TensorOptions().dtype(torch::kUInt8).device(weight.device());
    auto f16 = torch::TensorOptions().dtype(torch::kHalf).device(weight.device());
    auto packed = torch::empty({d_out, d_in / 2}, u8);
    auto scales = torch::empty({d_out, d_in / 128}, f16);
    auto zeros = torch::empty({d_out, d_in / 128}, f16);
    torch::Tensor copy;
    if (with_copy) copy = weight.clone();
    check_status(dq_quantize(h16(weight), static_cast<int32_t>(d_out), static_cast<int32_t>(d_in),
                             reinterpret_cast<uint8_t*>(packed.data_ptr()), h16m(scales), h16m(zeros),
                             stream_of(weight)),
                 "quantize_weights");
    return {packed, scales, zeros, copy};
}

// build_colmajor(weight [d_out, d_in] f16) -> mirror [d_in, d_out] f16 (contiguous)
torch::Tensor build_colmajor(const torch::Tensor& weight) {
    check_fp16_contiguous(weight, "weight");
    TORCH_CHECK(weight.dim() == 2, "weight must be 2D [d_out, d_in]");
    const int64_t d_out = weight.size(0), d_in = weight.size(1);
    TORCH_CHECK(d_in % 128 == 0, "d_in must be divisible by GROUP_SIZE=", 128);
    const at::cuda::CUDAGuard guard(weight.device());
    auto cm = torch::empty({d_in, d_out}, weight.options());
    check_status(dq_build_colmajor(h16(weight), static_cast<int32_t>(d_out),
                                   static_cast<int32_t>(d_in), h16m(cm), stream_of(weight)),
                 "build_colmajor");
    return cm;
}

// split_gemv(packed, scales, zeros, fp16_weights, x, outlier_k) -> y [d_out] f16
torch::Tensor split_gemv(const torch::Tensor& packed, const torch::Tensor& scales,
                         const torch::Tensor& zeros, const torch::Tensor& fp16_w,
                         const torch::Tensor& x, double outlier_k,
                         const c10::optional<torch::Tensor>& native) {
    dq_weights_t w = make_weights(packed, scales, zeros, fp16_w, x, true, native);
    const at::cuda::CUDAGuard guard(x.device());
    auto y = torch::empty({w.d_out}, x.options());
    void* stream = stream_of(x);
    const size_t wsb = dq_workspace_bytes(w.d_out, w.d_in);
    auto ws = workspace_for(x.device(), stream, wsb);
    check_status(dq_split_gemv(&w, h16(x), h16m(y), static_cast<float>(outlier_k), ws.data_ptr(),
                               static_cast<size_t>(ws.numel()), stream),
                 "split_gemv");
    return y;
}

// split_gemv_batched(packed, scales, zeros, fp16_weights, x [m, d_in], outlier_k, native)
//   -> y [m, d_out] f16, 1 <= m <= 16: the split GEMV of every row of x.
torch::Tensor split_gemv_batched(const torch::Tensor& packed, const torch::Tensor& scales,
                                 const torch::Tensor& zeros, const torch::Tensor& fp16_w,
                                 const torch::Tensor& x, double outlier_k, const torch::Tensor& native) {
    check_fp16_contiguous(x, "x");
    TORCH_CHECK(x.dim() == 2, "x must be 2D [m, d_in]");
    TORCH_CHECK(fp16_w.dim() == 2 && x.size(1) == fp16_w.size(1), "x must be [m, d_in] with d_in=", fp16_w.size(1));
    const int64_t m = x.size(0);
    TORCH_CHECK(m >= 1 && m <= 16, "split_gemv_batched takes 1 to 16 rows, got ", m);
    dq_weights_t w = make_weights(packed, scales, zeros, fp16_w, x[0], true, native);
    TORCH_CHECK(w.native != nullptr, "split_gemv_batched needs the native layout (build_native)");
    const at::cuda::CUDAGuard guard(x.device());
    auto y = torch::empty({m, w.d_out}, x.options());
    void* stream = stream_of(x);
    const size_t wsb = dq_workspace_bytes_batched(w.d_out, w.d_in, static_cast<int32_t>(m));
    auto ws = workspace_for(x.device(), stream, wsb);
    check_status(dq_split_gemv_batched(&w, h16(x), h16m(y), static_cast<int32_t>(m), static_cast<float>(outlier_k),
                                       ws.data_ptr(), static_cast<size_t>(ws.numel()), stream),
                 "split_gemv_batched");
    return y;
}

// int4_gemv(packed, scales, zeros, fp16_weights, x) -> y [d_out] f16
torch::Tensor int4_gemv(const torch::Tensor& packed, const torch::Tensor& scales,
                        const torch::Tensor& zeros, const torch::Tensor& fp16_w,
                        const torch::Tensor& x, const c10::optional<torch::Tensor>& native) {
    dq_weights_t w = make_weights(packed, scales, zeros, fp16_w, x, false, native);
    const at::cuda::CUDAGuard guard(x.device());
    auto y = torch::empty({w.d_out}, x.options());
    void* stream = stream_of(x);
    const size_t wsb = dq_workspace_bytes(w.d_out, w.d_in);
    auto ws = workspace_for(x.device(), stream, wsb);
    check_status(dq_int4_gemv(&w, h16(x), h16m(y), ws.data_ptr(), static_cast<size_t>(ws.numel()), stream),
                 "int4_gemv");
    return y;
}

// build_native(packed, scales, zeros) -> the unit layout the GEMV kernels stream (uint8 tensor)
torch::Tensor build_native(const torch::Tensor& packed, const torch::Tensor& scales, const torch::Tensor& zeros) {
    check_fp16_contiguous(scales, "scales");
    check_fp16_contiguous(zeros, "zeros");
    TORCH_CHECK(packed.is_cuda() && packed.is_contiguous() && packed.scalar_type() == at::kByte && packed.dim() == 2,
                "packed must be a contiguous 2D CUDA uint8 tensor");
    const int64_t d_out = packed.size(0), d_in = packed.size(1) * 2;
    TORCH_CHECK(d_in % 128 == 0, "d_in must be divisible by 128");
    TORCH_CHECK(scales.numel() == d_out * (d_in / 128) && zeros.numel() == scales.numel(),
                "scales/zeros must hold d_out * d_in/128 values");
    const at::cuda::CUDAGuard guard(packed.device());
    const size_t bytes = dq_native_bytes(static_cast<int32_t>(d_out), static_cast<int32_t>(d_in));
    auto out = torch::empty({static_cast<int64_t>(bytes)}, packed.options());
    check_status(dq_build_native(reinterpret_cast<const uint8_t*>(packed.data_ptr()), h16(scales), h16(zeros),
                                 static_cast<int32_t>(d_out), static_cast<int32_t>(d_in),
                                 reinterpret_cast<uint8_t*>(out.data_ptr()), stream_of(packed)),
                 "build_native");
    return out;
}

// reference_gemv(fp16_weights, x) -> y [d_out] f16   (csrc/bindings.cpp:162-182)
torch::Tensor reference_gemv(const torch::Tensor& fp16_w, const torch::Tensor& x) {
    TORCH_CHECK(fp16_w.dim() == 2, "fp16_weights must be 2D");
    check_fp16_contiguous(fp16_w, "fp16_weights");
    check_fp16_contiguous(x, "x");
    const int64_t d_out = fp16_w.size(0), d_in = fp16_w.size(1);
    TORCH_CHECK(x.numel() == d_in, "x length must equal d_in");
    TORCH_CHECK(d_in % 128 == 0, "d_in must be divisible by 128");
    const at::cuda::CUDAGuard guard(x.device());
    auto y = torch::empty({d_out}, x.options());
    check_status(dq_reference_gemv(h16(fp16_w), h16(x), h16m(y), static_cast<int32_t>(d_out),
                                   static_cast<int32_t>(d_in), stream_of(x)),
                 "reference_gemv");
    return y;
}

// detect_outliers(x, k) -> (mask_words int32 [d_in/32], indices int32 [d_in/4],
//                           count int32 [1], stats f32 [4]); no host synchronisation.
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor>
detect_outliers(const torch::Tensor& x, double outlier_k) {
    check_fp16_contiguous(x, "x");
    const int64_t d_in = x.numel();
    TORCH_CHECK(d_in > 0 && d_in % 128 == 0, "x length must be a positive multiple of 128");
    const at::cuda::CUDAGuard guard(x.device());
    auto i32 = torch::TensorOptions().dtype(torch::kInt32).device(x.device());
    auto mask = torch::empty({d_in / 32}, i32);
    auto idx = torch::empty({d_in / 4}, i32);
    auto cnt = torch::empty({1}, i32);
    auto stats = torch::empty({4}, torch::TensorOptions().dtype(torch::kFloat32).device(x.device()));
    check_status(dq_detect_outliers(h16(x), static_cast<int32_t>(d_in), static_cast<float>(outlier_k),
                                    reinterpret_cast<uint32_t*>(mask.data_ptr()),
                                    reinterpret_cast<int32_t*>(idx.data_ptr()),
                                    reinterpret_cast<int32_t*>(cnt.data_ptr()),
                                    reinterpret_cast<float*>(stats.data_ptr()), stream_of(x)),
                 "detect_outliers");
    return {mask, idx, cnt, stats};
}

// The weights of one DynQuantLinear, checked once when the module's buffers are
// (re)assigned, so that each forward call only checks x before the launch.
// Holds references to the buffers, whose device addresses it keeps in a
// dq_weights_t; the Python module drops the handle whenever a buffer object
// changes (load_weight, load_state_dict, .to()).
class SplitLinear {
public:
    SplitLinear(const torch::Tensor& packed, const torch::Tensor& scales, const torch::Tensor& zeros,
                const torch::Tensor& fp16_w, const torch::Tensor& native, double outlier_k)
        : packed_(packed), scales_(scales), zeros_(zeros), fp16_w_(fp16_w), native_(native), k_(outlier_k) {
        TORCH_CHECK(fp16_w.dim() == 2, "fp16_weights must be 2D");
        const auto probe = torch::empty({fp16_w.size(1)}, fp16_w.options());  // stands for x in the checks
        w_ = make_weights(packed, scales, zeros, fp16_w, probe, true, native);
        TORCH_CHECK(w_.native != nullptr, "SplitLinear needs the native layout (build_native)");
        dev_ = fp16_w.device();
        wsb_ = dq_workspace_bytes(w_.d_out, w_.d_in);
    }

    // y [d_out] for x [d_in] or [1, d_in] (float16, contiguous, on the weights'
    // device); None for any other x, which the caller routes through the
    // general path (dtype conversion, batches).
    // out: optional float16 [d_out] tensor on the same device to write y into
    // (contiguous); y is returned either way.
    py::object forward(const torch::Tensor& x, const c10::optional<torch::Tensor>& out) {
        if (!x.is_cuda() || x.scalar_type() != at::kHalf || !x.is_contiguous() || x.numel() != w_.d_in ||
            x.dim() > 2 || x.device() != dev_)
            return py::none();
        const bool has_out = out.has_value() && out->defined();
        if (has_out && (!out->is_cuda() || out->scalar_type() != at::kHalf || !out->is_contiguous() ||
                        out->numel() != w_.d_out || out->device() != dev_))
            return py::none();
        torch::Tensor xa = (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15u) ? x.clone() : x;
        const at::cuda::CUDAGuard guard(dev_);
        auto y = has_out ? *out : torch::empty({w_.d_out}, x.options());
        void* stream = at::cuda::getCurrentCUDAStream().stream();
        auto ws = workspace_for(dev_, stream, wsb_);
        check_status(dq_split_gemv(&w_, h16(xa), h16m(y), static_cast<float>(k_), ws.data_ptr(),
                                   static_cast<size_t>(ws.numel()), stream),
                     "split_gemv");
        return py::cast(y);
    }

private:
    torch::Tensor packed_, scales_, zeros_, fp16_w_, native_;
    double k_;
    dq_weights_t w_{};
    torch::Device dev_{torch::kCPU};
    size_t wsb_ = 0;
};

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    py::class_<SplitLinear>(m, "SplitLinear")
        .def(py::init<const torch::Tensor&, const torch::Tensor&, const torch::Tensor&, const torch::Tensor&,
                      const torch::Tensor&, double>(),
             py::arg("packed"), py::arg("scales"), py::arg("zeros"), py::arg("fp16_weights"), py::arg("native"),
             py::arg("outlier_k"))
        .def("forward", &SplitLinear::forward, py::arg("x"), py::arg("out") = py::none());
    m.def("quantize_weights", &quantize_weights, "Quantize FP16 weight matrix to INT4 packed format",
          py::arg("weight"), py::arg("with_copy") = true);
    m.def("split_gemv", &split_gemv, "Fused dynamic-precision GEMV with runtime outlier detection",
          py::arg("packed"), py::arg("scales"), py::arg("zeros"), py::arg("fp16_weights"), py::arg("x"),
          py::arg("outlier_k"), py::arg("native") = py::none());
    m.def("split_gemv_batched", &split_gemv_batched, "Split GEMV of 1 to 16 activation vectors",
          py::arg("packed"), py::arg("scales"), py::arg("zeros"), py::arg("fp16_weights"), py::arg("x"),
          py::arg("outlier_k"), py::arg("native"));
    m.def("int4_gemv", &int4_gemv, "Dense INT4 GEMV baseline", py::arg("packed"), py::arg("scales"),
          py::arg("zeros"), py::arg("fp16_weights"), py::arg("x"), py::arg("native") = py::none());
    m.def("build_native", &build_native, "Unit layout streamed by the GEMV kernels");
    m.def("reference_gemv", &reference_gemv, "FP16 dense reference GEMV");
    m.def("build_colmajor", &build_colmajor, "Column-major FP16 mirror of a weight matrix");
    m.def("detect_outliers", &detect_outliers, "Standalone outlier detector");
    m.def("version", []() { return dq_version(); });
    m.def("reset_workspaces", &reset_workspaces, "Zero the cached GEMV workspaces");
    m.def("read_device_error", [](bool clear) {
        uint32_t w = 0;
        check_status(dq_read_device_error(&w, clear ? 1 : 0), "read_device_error");
        return w;
    }, py::arg("clear") = false);
}
