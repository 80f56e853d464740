// The replica path's entry points as torch custom operators (namespace p2p_b200), over the C ABI of
// include/p2p_b200.h: torch tensors in and out, launches on the current CUDA stream, errors as c10::Error (RuntimeError
// in Python). Each op has a Meta kernel, so the dispatcher, torch.library fake tensors and shape propagation see it.
//
// The reference binds its GPU kernel the same way, as a torch extension op (p2p/compact.cu:265-293, spmm). The C ABI
// symbols are resolved from libp2p_b200.so, which p2pllm_b200._lib loads into the global scope first.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "p2p_b200.h"

namespace {

int dtype_code(const at::Tensor& t) {
    switch (t.scalar_type()) {
        case at::kBFloat16: return P2P_BF16;
        case at::kHalf: return P2P_F16;
        case at::kFloat: return P2P_F32;
        default: TORCH_CHECK(false, "p2p_b200: bfloat16, float16 or float32, got ", t.scalar_type());
    }
    return -1;
}

void check(int status, const char* what) {
    TORCH_CHECK(status == P2P_OK, what, ": ", p2p_last_error(), " (status ", status, ")");
}

void* stream_of(const at::Tensor& t) {
    return reinterpret_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

// A zeroed scratch buffer per device, purpose and stream, kept for the process (the kernels leave it zeroed again;
// launches on one stream run in order and may share it, launches on two streams may overlap and must not).
std::mutex ws_mu;
std::map<std::tuple<int, int, void*>, at::Tensor> ws_cache;

void* workspace(const at::Tensor& like, size_t bytes, int purpose) {
    if (bytes == 0) return nullptr;
    auto& cache = ws_cache;
    std::lock_guard<std::mutex> lock(ws_mu);
    const auto key = std::make_tuple((int)like.device().index(), purpose, stream_of(like));
    auto it = cache.find(key);
    if (it == cache.end() || (size_t)it->second.numel() < bytes) {
        const int64_t n = (int64_t)std::max(bytes, (size_t)1 << 20);
        cache[key] = at::zeros({n}, like.options().dtype(at::kByte));
        it = cache.find(key);
    }
    return it->second.data_ptr();
}

// Zeroes every cached workspace of `device` (after a launch gave up, which may leave ticket counters taken).
void zero_workspaces(int64_t device) {
    std::lock_guard<std::mutex> lock(ws_mu);
    for (auto& [key, ws] : ws_cache) {
        if (std::get<0>(key) != (int)device) continue;
        const c10::cuda::CUDAGuard guard(ws.device());
        ws.zero_();
    }
}

// x as the GEMMs take it: 2-D, unit column stride, 16-byte aligned rows.
at::Tensor gemm_input(const at::Tensor& x, int64_t cols) {
    TORCH_CHECK(x.is_cuda(), "p2p_b200: CUDA tensors only (the replica path has no CPU fallback)");
    TORCH_CHECK(x.dim() == 2 && x.size(1) == cols, "p2p_b200: x of ", x.sizes(), " does not have ", cols, " columns");
    if (x.stride(1) == 1 && x.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0) return x;
    at::Tensor c = x.contiguous();
    return reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 == 0 ? c : c.clone();
}

void check_out(const at::Tensor& out, const at::Tensor& x, int64_t rows) {
    TORCH_CHECK(out.is_cuda() && out.device() == x.device() && out.scalar_type() == x.scalar_type() && out.dim() == 2 &&
                    out.size(0) == x.size(0) && out.size(1) == rows && (out.stride(1) == 1 || out.numel() == 0),
                "p2p_b200: out of ", out.sizes(), " does not take y [", x.size(0), ", ", rows, "]");
}

// ---- the compact GEMM, tensor-core layout (values + positions) -------------------------------------------------------

void spmm_tc_into(const at::Tensor& x_in, const at::Tensor& words, const at::Tensor& seg, int64_t rows, int64_t cols,
                  int64_t seg_cap, const at::Tensor& out) {
    const c10::cuda::CUDAGuard guard(x_in.device());
    const at::Tensor x = gemm_input(x_in, cols);
    check_out(out, x, rows);
    const size_t need = p2p_spmm_tc_workspace(rows, cols, x.size(0));
    check(p2p_spmm_tc(x.data_ptr(), dtype_code(x), x.size(0), cols, x.stride(0),
                      reinterpret_cast<const uint32_t*>(words.data_ptr()), seg.data_ptr<int64_t>(), rows, seg_cap,
                      out.data_ptr(), out.stride(0), workspace(x, need, 0), need, stream_of(x)),
          "p2p_spmm_tc");
}

at::Tensor spmm_tc(const at::Tensor& x, const at::Tensor& words, const at::Tensor& seg, int64_t rows, int64_t cols,
                   int64_t seg_cap) {
    at::Tensor out = at::empty({x.size(0), rows}, x.options());
    spmm_tc_into(x, words, seg, rows, cols, seg_cap, out);
    return out;
}

// ---- the compact GEMM, bitmask layout ------------------------------------------------------------------------------

void spmm_mask_into(const at::Tensor& x_in, const at::Tensor& data, const at::Tensor& seg, int64_t rows, int64_t cols,
                    const at::Tensor& out) {
    const c10::cuda::CUDAGuard guard(x_in.device());
    const at::Tensor x = gemm_input(x_in, cols);
    check_out(out, x, rows);
    const size_t need = p2p_spmm_mask_workspace(rows, cols, x.size(0));
    check(p2p_spmm_mask(x.data_ptr(), dtype_code(x), x.size(0), cols, x.stride(0), data.data_ptr(),
                        seg.data_ptr<int64_t>(), rows, out.data_ptr(), out.stride(0), workspace(x, need, 1), need,
                        stream_of(x)),
          "p2p_spmm_mask");
}

at::Tensor spmm_mask(const at::Tensor& x, const at::Tensor& data, const at::Tensor& seg, int64_t rows, int64_t cols) {
    at::Tensor out = at::empty({x.size(0), rows}, x.options());
    spmm_mask_into(x, data, seg, rows, cols, out);
    return out;
}

at::Tensor gemm_meta(const at::Tensor& x, int64_t rows) { return at::empty({x.size(0), rows}, x.options()); }
at::Tensor spmm_tc_meta(const at::Tensor& x, const at::Tensor&, const at::Tensor&, int64_t rows, int64_t, int64_t) {
    return gemm_meta(x, rows);
}
at::Tensor spmm_mask_meta(const at::Tensor& x, const at::Tensor&, const at::Tensor&, int64_t rows, int64_t) {
    return gemm_meta(x, rows);
}
void spmm_tc_into_meta(const at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t, int64_t, int64_t,
                       const at::Tensor&) {}
void spmm_mask_into_meta(const at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t, int64_t, const at::Tensor&) {}

// ---- calibration, combine, parts ------------------------------------------------------------------------------------

void sumsq_cols(const at::Tensor& x_in, const at::Tensor& sums) {
    TORCH_CHECK(x_in.is_cuda() && sums.is_cuda(), "p2p_b200: CUDA tensors only");
    const c10::cuda::CUDAGuard guard(x_in.device());
    at::Tensor x = x_in.reshape({-1, x_in.size(-1)});
    if (x.stride(-1) != 1) x = x.contiguous();
    TORCH_CHECK(sums.scalar_type() == at::kDouble && sums.numel() == x.size(1) && sums.is_contiguous(),
                "p2p_b200: sums must be a contiguous float64 vector of x's columns");
    const size_t need = p2p_sumsq_workspace(x.size(0), x.size(1), dtype_code(x));
    check(p2p_sumsq_cols(x.data_ptr(), dtype_code(x), x.size(0), x.size(1), x.stride(0), sums.data_ptr<double>(),
                         workspace(x, need, 2), need, stream_of(x)),
          "p2p_sumsq_cols");
}

std::vector<at::Tensor> same_shape(const at::TensorList& ts, const at::Tensor& ref) {
    std::vector<at::Tensor> out;
    for (const at::Tensor& t : ts) {
        TORCH_CHECK(t.is_cuda() && t.sizes() == ref.sizes() && t.scalar_type() == ref.scalar_type(),
                    "p2p_b200: part of ", t.sizes(), " differs from ", ref.sizes());
        out.push_back(t.contiguous());
    }
    return out;
}

at::Tensor combine(at::TensorList parts, const at::Tensor& h, const at::Tensor& h_copy) {
    const c10::cuda::CUDAGuard guard(h.device());
    const std::vector<at::Tensor> ps = same_shape(parts, h);
    const std::vector<at::Tensor> hs = same_shape({h, h_copy}, h);
    std::vector<const void*> ptrs;
    for (const at::Tensor& p : ps) ptrs.push_back(p.data_ptr());
    at::Tensor out = at::empty_like(hs[0], at::MemoryFormat::Contiguous);
    check(p2p_combine(ptrs.data(), (int)ptrs.size(), hs[0].data_ptr(), hs[1].data_ptr(), out.data_ptr(),
                      dtype_code(out), out.numel(), stream_of(out)),
          "p2p_combine");
    return out;
}

at::Tensor sum_parts(at::TensorList parts) {
    TORCH_CHECK(!parts.empty(), "p2p_b200: no parts");
    const c10::cuda::CUDAGuard guard(parts[0].device());
    const std::vector<at::Tensor> ps = same_shape(parts, parts[0]);
    std::vector<const void*> ptrs;
    for (const at::Tensor& p : ps) ptrs.push_back(p.data_ptr());
    at::Tensor out = at::empty_like(ps[0], at::MemoryFormat::Contiguous);
    check(p2p_sum_parts(ptrs.data(), (int)ptrs.size(), out.data_ptr(), dtype_code(out), out.numel(), stream_of(out)),
          "p2p_sum_parts");
    return out;
}

at::Tensor combine_meta(at::TensorList, const at::Tensor& h, const at::Tensor&) {
    return at::empty_like(h, at::MemoryFormat::Contiguous);
}
at::Tensor sum_parts_meta(at::TensorList parts) { return at::empty_like(parts[0], at::MemoryFormat::Contiguous); }
void sumsq_cols_meta(const at::Tensor&, const at::Tensor&) {}

}  // namespace

TORCH_LIBRARY(p2p_b200, m) {
    m.def("spmm_tc(Tensor x, Tensor words, Tensor seg, int rows, int cols, int seg_cap) -> Tensor");
    m.def("spmm_tc_into(Tensor x, Tensor words, Tensor seg, int rows, int cols, int seg_cap, Tensor(a!) out) -> ()");
    m.def("spmm_mask(Tensor x, Tensor data, Tensor seg, int rows, int cols) -> Tensor");
    m.def("spmm_mask_into(Tensor x, Tensor data, Tensor seg, int rows, int cols, Tensor(a!) out) -> ()");
    m.def("sumsq_cols(Tensor x, Tensor(a!) sums) -> ()");
    m.def("combine(Tensor[] parts, Tensor h, Tensor h_copy) -> Tensor");
    m.def("sum_parts(Tensor[] parts) -> Tensor");
    m.def("zero_workspaces(int device) -> ()", &zero_workspaces);
}

TORCH_LIBRARY_IMPL(p2p_b200, CUDA, m) {
    m.impl("spmm_tc", &spmm_tc);
    m.impl("spmm_tc_into", &spmm_tc_into);
    m.impl("spmm_mask", &spmm_mask);
    m.impl("spmm_mask_into", &spmm_mask_into);
    m.impl("sumsq_cols", &sumsq_cols);
    m.impl("combine", &combine);
    m.impl("sum_parts", &sum_parts);
}

TORCH_LIBRARY_IMPL(p2p_b200, Meta, m) {
    m.impl("spmm_tc", &spmm_tc_meta);
    m.impl("spmm_tc_into", &spmm_tc_into_meta);
    m.impl("spmm_mask", &spmm_mask_meta);
    m.impl("spmm_mask_into", &spmm_mask_into_meta);
    m.impl("sumsq_cols", &sumsq_cols_meta);
    m.impl("combine", &combine_meta);
    m.impl("sum_parts", &sum_parts_meta);
}
