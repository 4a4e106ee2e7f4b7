// PyTorch operator layer: registers the reference's op schemas (torchsoftdtw::forward / backward,
// src/torchsoftdtw/csrc/softdtw.cpp:342-345) and this library's fused squared-L2 ops
// (torchsoftdtw_b200::l2_forward / l2_backward), and forwards every call to the C ABI of
// libsdtw_b200.so (include/sdtw_b200.h). No kernel runs here, and there is no CPU implementation:
// CPU tensors are validated (so argument errors read exactly as the reference's) and then rejected.
//
// Built against the regular (non-stable) libtorch API: with the stable ABI, a C++ exception thrown
// from a boxed kernel crashes the process under torch 2.11 instead of surfacing as RuntimeError.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cstdlib>
#include <mutex>
#include <tuple>
#include <unordered_map>

#include "sdtw_b200.h"

namespace {

using at::Tensor;

// softdtw.cpp:301-323, same conditions and messages.
void forward_checks(const Tensor& D, const Tensor& lengths_x, const Tensor& lengths_y, double gamma)
{
    TORCH_CHECK(D.dim() == 3, "D must be 3D (B, N, M)");
    TORCH_CHECK(lengths_x.dim() == 1 && lengths_y.dim() == 1, "lengths must be 1D");
    TORCH_CHECK(D.size(0) == lengths_x.size(0) && D.size(0) == lengths_y.size(0), "Batch size mismatch");
    TORCH_CHECK(gamma > 0, "gamma must be positive");
    const auto st = D.scalar_type();
    TORCH_CHECK(st == at::kFloat || st == at::kDouble || st == at::kHalf || st == at::kBFloat16,
                "D must be float16, bfloat16, float32 or float64");
    const auto lx = lengths_x.scalar_type(), ly = lengths_y.scalar_type();
    TORCH_CHECK(lx == at::kInt || lx == at::kLong, "lengths_x must be int32 or int64");
    TORCH_CHECK(ly == at::kInt || ly == at::kLong, "lengths_y must be int32 or int64");
}

void cuda_only(const Tensor& t)
{
    TORCH_CHECK(false, "torchsoftdtw_b200 runs on CUDA devices only (sm_100); got a tensor on ", t.device(),
                ". There is no CPU implementation.");
}

void same_device(const Tensor& ref, const Tensor& t, const char* name)
{
    TORCH_CHECK(t.device() == ref.device(), name, " must be on the same device as D (", ref.device(), "), got ",
                t.device());
}

at::ScalarType acc_type(at::ScalarType st)
{
    return (st == at::kHalf || st == at::kBFloat16) ? at::kFloat : st;
}

sdtw_dtype code_of(at::ScalarType st) { return st == at::kDouble ? SDTW_F64 : SDTW_F32; }

// Lengths as the kernels read them: int32 or int64, contiguous, on D's device.
// The kernels read both length arrays with one element type: when lengths_x and lengths_y differ (one int32,
// one int64) both go to int64, as the reference converts each to int64 (softdtw.cpp:67-70).
Tensor prep_lengths(const Tensor& l, const Tensor& other)
{
    return l.scalar_type() == other.scalar_type() ? l.contiguous() : l.to(at::kLong).contiguous();
}

// One sticky device error word per device, owned by this library for the process lifetime. It is created
// by the first op call on the device, which must not be under CUDA-graph capture: a word allocated there
// would come from the graph's private memory pool (and its zero-fill would be a captured memset), and the
// library would keep a pointer that dies with the graph. A capture that reaches a device without a word
// raises instead; one eager call before the capture (a warm-up step) creates it.
uint32_t* error_word(const Tensor& like)
{
    static std::mutex mu;
    static std::unordered_map<int, Tensor> words;
    std::lock_guard<std::mutex> lock(mu);
    const int dev = like.get_device();
    auto it = words.find(dev);
    if (it == words.end()) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        const cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev).stream();
        TORCH_CHECK(cudaStreamIsCapturing(stream, &cap) == cudaSuccess && cap == cudaStreamCaptureStatusNone,
                    "torchsoftdtw_b200: the first op call on ", like.device(),
                    " is under CUDA-graph capture; run one call outside the capture first (a warm-up step), "
                    "which creates the device's error word");
        it = words.emplace(dev, at::zeros({1}, like.options().dtype(at::kInt))).first;
    }
    return reinterpret_cast<uint32_t*>(it->second.data_ptr<int>());
}

bool sync_checks_enabled()
{
    static const bool on = [] {
        const char* v = std::getenv("TORCHSOFTDTW_B200_SYNC_CHECK");
        return v && v[0] && v[0] != '0';
    }();
    return on;
}

void check_status(sdtw_status st, const char* what)
{
    TORCH_CHECK(st == SDTW_OK, "torchsoftdtw_b200 ", what, " failed: ", sdtw_status_string(st));
}

// With TORCHSOFTDTW_B200_SYNC_CHECK=1, every op synchronises and raises on a device-side error.
void maybe_sync_check(const Tensor& like, cudaStream_t stream)
{
    if (!sync_checks_enabled()) return;
    const uint32_t bits = sdtw_read_error_word(error_word(like), stream);
    TORCH_CHECK(bits == 0, "torchsoftdtw_b200 device error bits 0x", std::hex, bits,
                (bits & SDTW_ERR_TIMEOUT) ? " (a wait on a neighbouring strip timed out)" : "",
                (bits & SDTW_ERR_BAD_LENGTH) ? " (a length was outside [0, N] / [0, M])" : "");
}

// band_r: R is read by this library's backward alone (the module path), which needs only part of it.
std::tuple<Tensor, Tensor> run_forward(const Tensor& Dacc, const Tensor& lx, const Tensor& ly, double gamma,
                                       int64_t bandwidth, bool band_r = false)
{
    const int64_t B = Dacc.size(0), N = Dacc.size(1), M = Dacc.size(2);
    const auto st = Dacc.scalar_type();
    auto opts = Dacc.options();
    Tensor R = at::empty({B, N + 2, M + 2}, opts);
    Tensor costs = at::empty({B}, opts);
    const size_t wsb = sdtw_forward_workspace_bytes(B, N, M, code_of(st));
    Tensor ws = at::empty({static_cast<int64_t>(wsb)}, opts.dtype(at::kByte));
    cudaStream_t stream = at::cuda::getCurrentCUDAStream(Dacc.get_device()).stream();
    check_status((band_r ? sdtw_forward_band_r : sdtw_forward)(code_of(st), Dacc.data_ptr(), B, N, M, lx.data_ptr(),
                                                              ly.data_ptr(), lx.scalar_type() == at::kInt, gamma,
                                                              bandwidth, R.data_ptr(), costs.data_ptr(), ws.data_ptr(),
                                                              wsb, error_word(Dacc), stream),
                 "forward");
    maybe_sync_check(Dacc, stream);
    return {costs, R};
}

Tensor run_backward(const Tensor& Racc, const Tensor& lx, const Tensor& ly, double gamma, int64_t bandwidth,
                    int64_t N, int64_t M)
{
    const int64_t B = Racc.size(0);
    const auto st = Racc.scalar_type();
    auto opts = Racc.options();
    Tensor E = at::empty({B, N, M}, opts);
    const size_t wsb = sdtw_backward_workspace_bytes(B, N, M, code_of(st));
    Tensor ws = at::empty({static_cast<int64_t>(wsb)}, opts.dtype(at::kByte));
    cudaStream_t stream = at::cuda::getCurrentCUDAStream(Racc.get_device()).stream();
    check_status(sdtw_backward(code_of(st), nullptr, Racc.data_ptr(), B, N, M, lx.data_ptr(), ly.data_ptr(),
                               lx.scalar_type() == at::kInt, gamma, bandwidth, E.data_ptr(), ws.data_ptr(), wsb,
                               error_word(Racc), stream),
                 "backward");
    maybe_sync_check(Racc, stream);
    return E;
}

// ---------------------------------------------------------------------------------------------------
// torchsoftdtw::forward / backward
// ---------------------------------------------------------------------------------------------------
std::tuple<Tensor, Tensor> forward_cuda(const Tensor& D, const Tensor& lengths_x, const Tensor& lengths_y,
                                        double gamma, int64_t bandwidth)
{
    forward_checks(D, lengths_x, lengths_y, gamma);
    same_device(D, lengths_x, "lengths_x");
    same_device(D, lengths_y, "lengths_y");
    const c10::cuda::CUDAGuard guard(D.device());
    const Tensor Dacc = D.to(acc_type(D.scalar_type())).contiguous();
    return run_forward(Dacc, prep_lengths(lengths_x, lengths_y), prep_lengths(lengths_y, lengths_x), gamma, bandwidth);
}

Tensor backward_cuda(const Tensor& D, const Tensor& R, const Tensor& lengths_x, const Tensor& lengths_y,
                     double gamma, int64_t bandwidth)
{
    forward_checks(D, lengths_x, lengths_y, gamma);
    const int64_t B = D.size(0), N = D.size(1), M = D.size(2);
    TORCH_CHECK(R.dim() == 3 && R.size(0) == B && R.size(1) == N + 2 && R.size(2) == M + 2,
                "R must have shape (B, N+2, M+2) = (", B, ", ", N + 2, ", ", M + 2, "), got ", R.sizes());
    same_device(D, R, "R");
    same_device(D, lengths_x, "lengths_x");
    same_device(D, lengths_y, "lengths_y");
    const c10::cuda::CUDAGuard guard(D.device());
    const auto acc = acc_type(D.scalar_type());
    const Tensor Racc = R.to(acc).contiguous();
    Tensor E = run_backward(Racc, prep_lengths(lengths_x, lengths_y), prep_lengths(lengths_y, lengths_x), gamma, bandwidth, N, M);
    if (E.scalar_type() != D.scalar_type()) E = E.to(D.scalar_type());
    return E;
}

std::tuple<Tensor, Tensor> forward_cpu(const Tensor& D, const Tensor& lengths_x, const Tensor& lengths_y,
                                       double gamma, int64_t bandwidth)
{
    (void)bandwidth;
    forward_checks(D, lengths_x, lengths_y, gamma);
    cuda_only(D);
    return {};
}

Tensor backward_cpu(const Tensor& D, const Tensor& R, const Tensor& lengths_x, const Tensor& lengths_y, double gamma,
                    int64_t bandwidth)
{
    (void)R;
    (void)bandwidth;
    forward_checks(D, lengths_x, lengths_y, gamma);
    cuda_only(D);
    return {};
}

// ---------------------------------------------------------------------------------------------------
// torchsoftdtw_b200::l2_forward / l2_backward — the SoftDTW module's squared-L2 path
// ---------------------------------------------------------------------------------------------------
void xy_checks(const Tensor& X, const Tensor& Y, const Tensor& lengths_x, const Tensor& lengths_y, double gamma)
{
    TORCH_CHECK(X.dim() == 3 && Y.dim() == 3, "X and Y must be 3D (B, N, d) and (B, M, d)");
    TORCH_CHECK(X.size(0) == Y.size(0), "Batch size mismatch between X and Y");
    TORCH_CHECK(X.size(2) == Y.size(2), "X and Y must have the same feature dimension");
    TORCH_CHECK(lengths_x.dim() == 1 && lengths_y.dim() == 1, "lengths must be 1D");
    TORCH_CHECK(X.size(0) == lengths_x.size(0) && X.size(0) == lengths_y.size(0), "Batch size mismatch");
    TORCH_CHECK(gamma > 0, "gamma must be positive");
    const auto st = X.scalar_type();
    TORCH_CHECK(st == at::kFloat || st == at::kDouble || st == at::kHalf || st == at::kBFloat16,
                "X must be float16, bfloat16, float32 or float64");
    TORCH_CHECK(Y.scalar_type() == st, "X and Y must have the same dtype");
    const auto lx = lengths_x.scalar_type(), ly = lengths_y.scalar_type();
    TORCH_CHECK(lx == at::kInt || lx == at::kLong, "lengths_x must be int32 or int64");
    TORCH_CHECK(ly == at::kInt || ly == at::kLong, "lengths_y must be int32 or int64");
    TORCH_CHECK(X.is_cuda(), "torchsoftdtw_b200 runs on CUDA devices only (sm_100); got a tensor on ", X.device());
    same_device(X, Y, "Y");
    same_device(X, lengths_x, "lengths_x");
    same_device(X, lengths_y, "lengths_y");
}

// The module path's R: the forward's strip tiles (B, S, NBt, 32, 32) when both wavefront directions run on
// the pair-resident kernels for this shape (sdtw_r_tiled), else the padded R (B, N+2, M+2) of the op. The
// backward tells the two apart by the number of dimensions.
std::tuple<Tensor, Tensor> run_forward_module(const Tensor& Dacc, const Tensor& lx, const Tensor& ly, double gamma,
                                              int64_t bandwidth)
{
    const int64_t B = Dacc.size(0), N = Dacc.size(1), M = Dacc.size(2);
    const auto st = Dacc.scalar_type();
    if (B == 0 || N == 0 || M == 0 || !sdtw_r_tiled(B, N, M, code_of(st)))
        return run_forward(Dacc, lx, ly, gamma, bandwidth, true);
    auto opts = Dacc.options();
    const int64_t S = (N + 31) / 32, NBt = sdtw_r_tiles_elems(1, 32, M) / 1024;
    Tensor Rt = at::empty({B, S, NBt, 32, 32}, opts);
    Tensor costs = at::empty({B}, opts);
    const size_t wsb = sdtw_forward_workspace_bytes(B, N, M, code_of(st));
    Tensor ws = at::empty({static_cast<int64_t>(wsb)}, opts.dtype(at::kByte));
    cudaStream_t stream = at::cuda::getCurrentCUDAStream(Dacc.get_device()).stream();
    check_status(sdtw_forward_tiles(code_of(st), Dacc.data_ptr(), B, N, M, lx.data_ptr(), ly.data_ptr(),
                                    lx.scalar_type() == at::kInt, gamma, bandwidth, Rt.data_ptr(), costs.data_ptr(),
                                    ws.data_ptr(), wsb, error_word(Dacc), stream),
                 "forward");
    maybe_sync_check(Dacc, stream);
    return {costs, Rt};
}

Tensor run_backward_module(const Tensor& Racc, const Tensor& lx, const Tensor& ly, double gamma, int64_t bandwidth,
                           int64_t N, int64_t M)
{
    if (Racc.dim() != 5) return run_backward(Racc, lx, ly, gamma, bandwidth, N, M);
    const int64_t B = Racc.size(0);
    const auto st = Racc.scalar_type();
    auto opts = Racc.options();
    Tensor E = at::empty({B, N, M}, opts);
    const size_t wsb = sdtw_backward_workspace_bytes(B, N, M, code_of(st));
    Tensor ws = at::empty({static_cast<int64_t>(wsb)}, opts.dtype(at::kByte));
    cudaStream_t stream = at::cuda::getCurrentCUDAStream(Racc.get_device()).stream();
    check_status(sdtw_backward_tiles(code_of(st), Racc.data_ptr(), B, N, M, lx.data_ptr(), ly.data_ptr(),
                                     lx.scalar_type() == at::kInt, gamma, bandwidth, E.data_ptr(), ws.data_ptr(), wsb,
                                     error_word(Racc), stream),
                 "backward");
    maybe_sync_check(Racc, stream);
    return E;
}

// True when the fused forward (cost tiles computed inside the wavefront, sdtw_forward_l2_tiles) runs this
// problem: TORCHSOFTDTW_B200_FUSED_COST=1 in the environment (read on every call, as the FakeTensor kernel
// does), fp32 arithmetic and a shape the library accepts (sdtw_forward_l2_fused_ok). It trades the cost
// matrix's memory (B N M values) for in-wavefront products on the warp tensor-core path, which at d = 64
// makes the forward slower than the stored-D pair of kernels; hence off by default. The operands are
// contiguous accumulation-type copies, so their alignment is the allocator's (checked anyway).
bool l2_fused(const Tensor& Xc, const Tensor& Yc)
{
    const char* env = std::getenv("TORCHSOFTDTW_B200_FUSED_COST");
    if (!env || !env[0] || env[0] == '0') return false;
    const int64_t B = Xc.size(0), N = Xc.size(1), M = Yc.size(1), d = Xc.size(2);
    return Xc.scalar_type() == at::kFloat && sdtw_forward_l2_fused_ok(B, N, M, d) &&
           reinterpret_cast<uintptr_t>(Xc.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(Yc.data_ptr()) % 16 == 0;
}

// Returns (costs, R, D, clamp_flags): R as run_forward_module returns it; D is the clamped cost matrix with
// the clamp recorded in its sign bit; clamp_flags (B,) int32 marks the pairs that have a clamped cell.
// When the fused forward runs (l2_fused), D is never formed: the third output is instead the clamp mask
// (B, N, ceil(M / 32)) int32, bit c % 32 of word c / 32 set where cell (i, c) was clamped, and R is the
// strip tiles.
std::tuple<Tensor, Tensor, Tensor, Tensor> l2_forward_cuda(const Tensor& X, const Tensor& Y,
                                                           const Tensor& lengths_x, const Tensor& lengths_y,
                                                           double gamma, int64_t bandwidth)
{
    xy_checks(X, Y, lengths_x, lengths_y, gamma);
    const c10::cuda::CUDAGuard guard(X.device());
    const auto acc = acc_type(X.scalar_type());
    const Tensor Xc = X.to(acc).contiguous(), Yc = Y.to(acc).contiguous();
    const int64_t B = Xc.size(0), N = Xc.size(1), M = Yc.size(1), d = Xc.size(2);
    if (B > 0 && N > 0 && M > 0 && l2_fused(Xc, Yc)) {
        const Tensor lx = prep_lengths(lengths_x, lengths_y), ly = prep_lengths(lengths_y, lengths_x);
        auto opts = Xc.options();
        const int64_t S = (N + 31) / 32, NBt = sdtw_r_tiles_elems(1, 32, M) / 1024;
        Tensor Rt = at::empty({B, S, NBt, 32, 32}, opts);
        Tensor costs = at::empty({B}, opts);
        Tensor mask = at::empty({B, N, (M + 31) / 32}, opts.dtype(at::kInt));
        Tensor flags = at::empty({B}, opts.dtype(at::kInt));
        const size_t wsb = sdtw_forward_workspace_bytes(B, N, M, SDTW_F32);
        Tensor ws = at::empty({static_cast<int64_t>(wsb)}, opts.dtype(at::kByte));
        cudaStream_t stream = at::cuda::getCurrentCUDAStream(X.get_device()).stream();
        check_status(sdtw_forward_l2_tiles(Xc.data_ptr<float>(), Yc.data_ptr<float>(), B, N, M, d, lx.data_ptr(),
                                           ly.data_ptr(), lx.scalar_type() == at::kInt, gamma, bandwidth,
                                           Rt.data_ptr(), costs.data_ptr<float>(),
                                           reinterpret_cast<uint32_t*>(mask.data_ptr<int>()), flags.data_ptr<int>(),
                                           ws.data_ptr(), wsb, error_word(Xc), stream),
                     "forward");
        maybe_sync_check(Xc, stream);
        return {costs, Rt, mask, flags};
    }
    Tensor D = at::empty({B, N, M}, Xc.options());
    Tensor flags = at::empty({B}, Xc.options().dtype(at::kInt));
    cudaStream_t stream = at::cuda::getCurrentCUDAStream(X.get_device()).stream();
    const Tensor lx = prep_lengths(lengths_x, lengths_y), ly = prep_lengths(lengths_y, lengths_x);
    if (bandwidth >= 0) {
        // With a band the wavefronts read only the band's cells of D: compute only the tiles that hold them.
        const size_t wsb = sdtw_pairwise_l2_band_workspace_bytes(B, N, M);
        Tensor ws = at::empty({static_cast<int64_t>(wsb)}, Xc.options().dtype(at::kByte));
        check_status(sdtw_pairwise_l2_band(code_of(acc), Xc.data_ptr(), Yc.data_ptr(), B, N, M, d, lx.data_ptr(),
                                           ly.data_ptr(), lx.scalar_type() == at::kInt, bandwidth, D.data_ptr(),
                                           flags.data_ptr<int>(), ws.data_ptr(), wsb, stream),
                     "pairwise_l2_band");
    } else {
        check_status(sdtw_pairwise_l2(code_of(acc), Xc.data_ptr(), Yc.data_ptr(), B, N, M, d, D.data_ptr(),
                                      flags.data_ptr<int>(), stream),
                     "pairwise_l2");
    }
    auto [costs, R] = run_forward_module(D, lx, ly, gamma, bandwidth);
    return {costs, R, D, flags};
}

// Gradients of sum_b grad_costs[b] * costs[b] w.r.t. X and Y (each skipped when not requested).
std::tuple<Tensor, Tensor> l2_backward_cuda(const Tensor& X, const Tensor& Y, const Tensor& D, const Tensor& R,
                                            const Tensor& clamp_flags, const Tensor& lengths_x,
                                            const Tensor& lengths_y, const Tensor& grad_costs, double gamma,
                                            int64_t bandwidth, bool need_x, bool need_y)
{
    xy_checks(X, Y, lengths_x, lengths_y, gamma);
    const c10::cuda::CUDAGuard guard(X.device());
    const auto acc = acc_type(X.scalar_type());
    const Tensor Xc = X.to(acc).contiguous(), Yc = Y.to(acc).contiguous();
    const int64_t B = Xc.size(0), N = Xc.size(1), M = Yc.size(1), d = Xc.size(2);
    // The fused forward's clamp mask in place of D (see l2_forward_cuda).
    const bool fused = D.scalar_type() == at::kInt;
    TORCH_CHECK(fused ? (D.sizes() == at::IntArrayRef({B, N, (M + 31) / 32}) && acc == at::kFloat)
                      : (D.sizes() == at::IntArrayRef({B, N, M}) && D.scalar_type() == acc),
                "D has the wrong shape or dtype");
    const bool tiled = R.dim() == 5 &&
                       R.sizes() == at::IntArrayRef({B, (N + 31) / 32, sdtw_r_tiles_elems(1, 32, M) / 1024, 32, 32});
    TORCH_CHECK((tiled || R.sizes() == at::IntArrayRef({B, N + 2, M + 2})) && R.scalar_type() == acc,
                "R has the wrong shape or dtype");
    const Tensor lx = prep_lengths(lengths_x, lengths_y), ly = prep_lengths(lengths_y, lengths_x);
    Tensor E = run_backward_module(R.contiguous(), lx, ly, gamma, bandwidth, N, M);
    const Tensor g = grad_costs.to(acc).contiguous();
    // Gradients that are not requested come back as empty tensors.
    Tensor gX = need_x ? at::empty({B, N, d}, Xc.options()) : at::empty({0}, X.options());
    Tensor gY = need_y ? at::empty({B, M, d}, Xc.options()) : at::empty({0}, Y.options());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream(X.get_device()).stream();
    TORCH_CHECK(clamp_flags.numel() == B && clamp_flags.scalar_type() == at::kInt, "clamp_flags must be (B,) int32");
    Tensor Dg = D, flags = clamp_flags.contiguous();
    if (fused) {
        // Fold the clamp into E; the gradient kernels then see no clamped pair (all-zero flags, so they never
        // read their D argument, here E itself, whose sign bits are clear anyway: E >= 0).
        const Tensor mask = D.contiguous();
        check_status(sdtw_apply_clamp_mask(E.data_ptr<float>(), reinterpret_cast<const uint32_t*>(mask.data_ptr<int>()),
                                           flags.data_ptr<int>(), B, N, M, stream),
                     "apply_clamp_mask");
        Dg = E;
        flags = at::zeros({B}, flags.options());
    }
    if (bandwidth >= 0) {
        // E is zero outside the lengths and the band: the contraction skips the chunks that hold none of it.
        check_status(sdtw_grad_l2_band(code_of(acc), Xc.data_ptr(), Yc.data_ptr(), Dg.contiguous().data_ptr(),
                                       E.data_ptr(), g.data_ptr(), flags.data_ptr<int>(), B, N, M, d, lx.data_ptr(),
                                       ly.data_ptr(), lx.scalar_type() == at::kInt, bandwidth,
                                       need_x ? gX.data_ptr() : nullptr, need_y ? gY.data_ptr() : nullptr, stream),
                     "grad_l2_band");
    } else {
        check_status(sdtw_grad_l2(code_of(acc), Xc.data_ptr(), Yc.data_ptr(), Dg.contiguous().data_ptr(), E.data_ptr(),
                                  g.data_ptr(), flags.data_ptr<int>(), B, N, M, d, need_x ? gX.data_ptr() : nullptr,
                                  need_y ? gY.data_ptr() : nullptr, stream),
                     "grad_l2");
    }
    if (need_x && gX.scalar_type() != X.scalar_type()) gX = gX.to(X.scalar_type());
    if (need_y && gY.scalar_type() != Y.scalar_type()) gY = gY.to(Y.scalar_type());
    return {gX, gY};
}

// ---------------------------------------------------------------------------------------------------
// torchsoftdtw_b200::dist_forward / dist_backward — the SoftDTW module's L1 (kind 1) and cosine (kind 2)
// paths: the cost matrix from X, Y in this library's kernels, then the same wavefront ops.
// ---------------------------------------------------------------------------------------------------
void kind_check(int64_t kind, double eps)
{
    TORCH_CHECK(kind == SDTW_DIST_L1 || kind == SDTW_DIST_COSINE, "distance kind must be 1 (l1) or 2 (cosine)");
    TORCH_CHECK(eps > 0, "eps must be positive");
}

// Returns (costs, R, D).
std::tuple<Tensor, Tensor, Tensor> dist_forward_cuda(const Tensor& X, const Tensor& Y, const Tensor& lengths_x,
                                                     const Tensor& lengths_y, double gamma, int64_t bandwidth,
                                                     int64_t kind, double eps)
{
    xy_checks(X, Y, lengths_x, lengths_y, gamma);
    kind_check(kind, eps);
    const c10::cuda::CUDAGuard guard(X.device());
    const auto acc = acc_type(X.scalar_type());
    const Tensor Xc = X.to(acc).contiguous(), Yc = Y.to(acc).contiguous();
    const int64_t B = Xc.size(0), N = Xc.size(1), M = Yc.size(1), d = Xc.size(2);
    Tensor D = at::empty({B, N, M}, Xc.options());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream(X.get_device()).stream();
    check_status(sdtw_pairwise_dist(code_of(acc), static_cast<int>(kind), Xc.data_ptr(), Yc.data_ptr(), B, N, M, d,
                                    eps, D.data_ptr(), stream),
                 "pairwise_dist");
    auto [costs, R] = run_forward(D, prep_lengths(lengths_x, lengths_y), prep_lengths(lengths_y, lengths_x), gamma, bandwidth,
                                  true);
    return {costs, R, D};
}

std::tuple<Tensor, Tensor> dist_backward_cuda(const Tensor& X, const Tensor& Y, const Tensor& D, const Tensor& R,
                                              const Tensor& lengths_x, const Tensor& lengths_y,
                                              const Tensor& grad_costs, double gamma, int64_t bandwidth,
                                              int64_t kind, double eps, bool need_x, bool need_y)
{
    xy_checks(X, Y, lengths_x, lengths_y, gamma);
    kind_check(kind, eps);
    const c10::cuda::CUDAGuard guard(X.device());
    const auto acc = acc_type(X.scalar_type());
    const Tensor Xc = X.to(acc).contiguous(), Yc = Y.to(acc).contiguous();
    const int64_t B = Xc.size(0), N = Xc.size(1), M = Yc.size(1), d = Xc.size(2);
    TORCH_CHECK(D.sizes() == at::IntArrayRef({B, N, M}) && D.scalar_type() == acc, "D has the wrong shape or dtype");
    TORCH_CHECK(R.sizes() == at::IntArrayRef({B, N + 2, M + 2}) && R.scalar_type() == acc,
                "R has the wrong shape or dtype");
    Tensor E = run_backward(R.contiguous(), prep_lengths(lengths_x, lengths_y), prep_lengths(lengths_y, lengths_x), gamma, bandwidth, N, M);
    const Tensor g = grad_costs.to(acc).contiguous();
    Tensor gX = need_x ? at::empty({B, N, d}, Xc.options()) : at::empty({0}, X.options());
    Tensor gY = need_y ? at::empty({B, M, d}, Xc.options()) : at::empty({0}, Y.options());
    const size_t ws_bytes = sdtw_grad_dist_workspace_bytes(B, M, code_of(acc));
    Tensor ws = at::empty({static_cast<int64_t>(ws_bytes)}, Xc.options().dtype(at::kByte));
    cudaStream_t stream = at::cuda::getCurrentCUDAStream(X.get_device()).stream();
    check_status(sdtw_grad_dist(code_of(acc), static_cast<int>(kind), Xc.data_ptr(), Yc.data_ptr(),
                                D.contiguous().data_ptr(), E.data_ptr(), g.data_ptr(), B, N, M, d, eps,
                                ws.data_ptr(), need_x ? gX.data_ptr() : nullptr, need_y ? gY.data_ptr() : nullptr,
                                stream),
                 "grad_dist");
    if (need_x && gX.scalar_type() != X.scalar_type()) gX = gX.to(X.scalar_type());
    if (need_y && gY.scalar_type() != Y.scalar_type()) gY = gY.to(Y.scalar_type());
    return {gX, gY};
}

// ---------------------------------------------------------------------------------------------------
// torchsoftdtw_b200::forward_x2 / backward_x2 — the compensated fp32 ops (R as R_hi + R_lo): the same
// arguments and validation as torchsoftdtw::forward / backward, float32 (or float16 / bfloat16, promoted) D.
// ---------------------------------------------------------------------------------------------------
std::tuple<Tensor, Tensor, Tensor> forward_x2_cuda(const Tensor& D, const Tensor& lengths_x, const Tensor& lengths_y,
                                                   double gamma, int64_t bandwidth)
{
    forward_checks(D, lengths_x, lengths_y, gamma);
    TORCH_CHECK(D.scalar_type() != at::kDouble, "the compensated ops take float32 (or float16 / bfloat16) D");
    TORCH_CHECK(D.is_cuda(), "torchsoftdtw_b200 runs on CUDA devices only (sm_100); got a tensor on ", D.device());
    same_device(D, lengths_x, "lengths_x");
    same_device(D, lengths_y, "lengths_y");
    const c10::cuda::CUDAGuard guard(D.device());
    const Tensor Dc = D.to(at::kFloat).contiguous();
    const Tensor lx = prep_lengths(lengths_x, lengths_y), ly = prep_lengths(lengths_y, lengths_x);
    const int64_t B = Dc.size(0), N = Dc.size(1), M = Dc.size(2);
    Tensor Rh = at::empty({B, N + 2, M + 2}, Dc.options());
    Tensor Rl = at::empty({B, N + 2, M + 2}, Dc.options());
    Tensor costs = at::empty({B}, Dc.options());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream(D.get_device()).stream();
    check_status(sdtw_forward_x2(Dc.data_ptr<float>(), B, N, M, lx.data_ptr(), ly.data_ptr(),
                                 lx.scalar_type() == at::kInt, gamma, bandwidth, Rh.data_ptr<float>(),
                                 Rl.data_ptr<float>(), costs.data_ptr<float>(), error_word(Dc), stream),
                 "forward_x2");
    maybe_sync_check(Dc, stream);
    return {costs, Rh, Rl};
}

Tensor backward_x2_cuda(const Tensor& D, const Tensor& R_hi, const Tensor& R_lo, const Tensor& lengths_x,
                        const Tensor& lengths_y, double gamma, int64_t bandwidth)
{
    forward_checks(D, lengths_x, lengths_y, gamma);
    TORCH_CHECK(D.scalar_type() != at::kDouble, "the compensated ops take float32 (or float16 / bfloat16) D");
    const int64_t B = D.size(0), N = D.size(1), M = D.size(2);
    for (const Tensor* R : {&R_hi, &R_lo})
        TORCH_CHECK(R->dim() == 3 && R->size(0) == B && R->size(1) == N + 2 && R->size(2) == M + 2 &&
                        R->scalar_type() == at::kFloat,
                    "R_hi and R_lo must be float32 (B, N+2, M+2) = (", B, ", ", N + 2, ", ", M + 2, "), got ",
                    R->sizes());
    same_device(D, R_hi, "R_hi");
    same_device(D, R_lo, "R_lo");
    same_device(D, lengths_x, "lengths_x");
    same_device(D, lengths_y, "lengths_y");
    const c10::cuda::CUDAGuard guard(D.device());
    const Tensor Rh = R_hi.contiguous(), Rl = R_lo.contiguous();
    const Tensor lx = prep_lengths(lengths_x, lengths_y), ly = prep_lengths(lengths_y, lengths_x);
    Tensor E = at::empty({B, N, M}, Rh.options());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream(D.get_device()).stream();
    check_status(sdtw_backward_x2(Rh.data_ptr<float>(), Rl.data_ptr<float>(), B, N, M, lx.data_ptr(), ly.data_ptr(),
                                  lx.scalar_type() == at::kInt, gamma, bandwidth, E.data_ptr<float>(), error_word(Rh),
                                  stream),
                 "backward_x2");
    maybe_sync_check(Rh, stream);
    if (E.scalar_type() != D.scalar_type()) E = E.to(D.scalar_type());
    return E;
}

Tensor error_bits(const Tensor& like)
{
    // Reads and clears the sticky device error word of like's device (synchronises the current stream).
    TORCH_CHECK(like.is_cuda(), "error_bits needs a CUDA tensor to name the device");
    const c10::cuda::CUDAGuard guard(like.device());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream(like.get_device()).stream();
    const uint32_t bits = sdtw_read_error_word(error_word(like), stream);
    return at::tensor({static_cast<int64_t>(bits)}, at::kLong);
}

}  // namespace

TORCH_LIBRARY(torchsoftdtw, m)
{
    m.def("forward(Tensor D, Tensor lengths_x, Tensor lengths_y, float gamma, int bandwidth) -> (Tensor, Tensor)");
    m.def("backward(Tensor D, Tensor R, Tensor lengths_x, Tensor lengths_y, float gamma, int bandwidth) -> Tensor");
}

TORCH_LIBRARY_IMPL(torchsoftdtw, CUDA, m)
{
    m.impl("forward", &forward_cuda);
    m.impl("backward", &backward_cuda);
}

TORCH_LIBRARY_IMPL(torchsoftdtw, CPU, m)
{
    m.impl("forward", &forward_cpu);
    m.impl("backward", &backward_cpu);
}

TORCH_LIBRARY(torchsoftdtw_b200, m)
{
    m.def("l2_forward(Tensor X, Tensor Y, Tensor lengths_x, Tensor lengths_y, float gamma, int bandwidth) "
          "-> (Tensor, Tensor, Tensor, Tensor)");
    m.def("l2_backward(Tensor X, Tensor Y, Tensor D, Tensor R, Tensor clamp_flags, Tensor lengths_x, "
          "Tensor lengths_y, Tensor grad_costs, float gamma, int bandwidth, bool need_x, bool need_y) "
          "-> (Tensor, Tensor)");
    m.def("dist_forward(Tensor X, Tensor Y, Tensor lengths_x, Tensor lengths_y, float gamma, int bandwidth, "
          "int kind, float eps) -> (Tensor, Tensor, Tensor)");
    m.def("dist_backward(Tensor X, Tensor Y, Tensor D, Tensor R, Tensor lengths_x, Tensor lengths_y, "
          "Tensor grad_costs, float gamma, int bandwidth, int kind, float eps, bool need_x, bool need_y) "
          "-> (Tensor, Tensor)");
    m.def("forward_x2(Tensor D, Tensor lengths_x, Tensor lengths_y, float gamma, int bandwidth) -> (Tensor, Tensor, Tensor)");
    m.def("backward_x2(Tensor D, Tensor R_hi, Tensor R_lo, Tensor lengths_x, Tensor lengths_y, float gamma, "
          "int bandwidth) -> Tensor");
    m.def("error_bits(Tensor like) -> Tensor");
}

TORCH_LIBRARY_IMPL(torchsoftdtw_b200, CUDA, m)
{
    m.impl("l2_forward", &l2_forward_cuda);
    m.impl("l2_backward", &l2_backward_cuda);
    m.impl("dist_forward", &dist_forward_cuda);
    m.impl("dist_backward", &dist_backward_cuda);
    m.impl("forward_x2", &forward_x2_cuda);
    m.impl("backward_x2", &backward_x2_cuda);
    m.impl("error_bits", &error_bits);
}
