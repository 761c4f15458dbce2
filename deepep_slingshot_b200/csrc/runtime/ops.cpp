// Torch bindings of the standalone sm_100a ops.
#include "ops.hpp"

#include <ATen/cuda/CUDAContext.h>
#include <cstring>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "../kernels/api.h"
#include "../kernels/permute.h"
#include "../kernels/gemm.h"
#include "../kernels/symmetric_ops.h"

namespace ep {

namespace {

// Host-mapped error page shared by the standalone ops (timeouts of bounded waits land here).
ErrorState* op_error_page(ErrorState** dev_ptr) {
    static ErrorState* host = nullptr;
    static ErrorState* dev = nullptr;
    if (host == nullptr) {
        TORCH_CHECK(cudaHostAlloc(reinterpret_cast<void**>(&host), sizeof(ErrorState), cudaHostAllocMapped) == cudaSuccess);
        std::memset(host, 0, sizeof(ErrorState));
        TORCH_CHECK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&dev), host, 0) == cudaSuccess);
    }
    *dev_ptr = dev;
    return host;
}

std::tuple<int, int, int, int> op_error_state(bool clear) {
    ErrorState* dev;
    ErrorState* h = op_error_page(&dev);
    auto r = std::make_tuple(h->code, h->peer, h->detail, h->rank);
    if (clear) std::memset(h, 0, sizeof(ErrorState));
    return r;
}

KernelStatus op_status(double timeout_s) {
    KernelStatus s{};
    op_error_page(&s.host_error);
    s.abort_flag = nullptr;
    s.timeout_ns = (uint64_t)(timeout_s * 1e9);
    return s;
}

// Grouped block-scaled FP8 GEMM (tcgen05): d[rows, n] = per-expert A x B_e^T with 1x128 / 128x128 scales.
torch::Tensor grouped_gemm_fp8(const torch::Tensor& a, const torch::Tensor& sa, const torch::Tensor& b, const torch::Tensor& sb,
                               const torch::Tensor& offsets, const std::optional<torch::Tensor>& counts, int num_sms,
                               double timeout_s, bool ue8m0) {
    TORCH_CHECK(a.is_cuda() && a.dim() == 2 && a.is_contiguous() && a.scalar_type() == torch::kFloat8_e4m3fn);
    TORCH_CHECK(b.dim() == 3 && b.is_contiguous() && b.scalar_type() == torch::kFloat8_e4m3fn);
    const int rows = (int)a.size(0), k = (int)a.size(1), E = (int)b.size(0), n = (int)b.size(1);
    TORCH_CHECK(b.size(2) == k && k % 128 == 0 && n % 128 == 0, "k and n must be multiples of 128");
    TORCH_CHECK(sa.scalar_type() == torch::kFloat32 && sa.is_contiguous() && sa.size(0) == rows && sa.size(1) == k / 128);
    TORCH_CHECK(sb.scalar_type() == torch::kFloat32 && sb.is_contiguous() && sb.size(0) == E && sb.size(1) == n / 128 &&
                sb.size(2) == k / 128);
    TORCH_CHECK(offsets.scalar_type() == torch::kInt32 && offsets.numel() == E + 1);
    if (counts.has_value()) TORCH_CHECK(counts->scalar_type() == torch::kInt32 && counts->numel() == E);
    auto d = torch::empty({rows, n}, a.options().dtype(torch::kBFloat16));
    if (num_sms <= 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    }
    GemmArgs g{};
    g.a = a.data_ptr();
    g.sa = sa.data_ptr<float>();
    g.b = b.data_ptr();
    g.sb = sb.data_ptr<float>();
    g.offsets = offsets.data_ptr<int>();
    g.expert_counts = counts.has_value() ? counts->data_ptr<int>() : nullptr;
    g.d = d.data_ptr();
    g.rows = rows;
    g.n = n;
    g.k = k;
    g.num_experts = E;
    g.block_scaled = ue8m0 ? 1 : 0;
    g.st = op_status(timeout_s);
    const int rc = launch_grouped_gemm_fp8(g, num_sms, at::cuda::getCurrentCUDAStream());
    TORCH_CHECK(rc == 0, "grouped_gemm_fp8 launch failed (code " + std::to_string(rc) + ")");
    return d;
}

// Masked grouped FP8 GEMM (tcgen05) over the low-latency per-expert padded layout:
// a [E, slots, k] e4m3, sa [E, slots, k/128] fp32 (any strides, e.g. the dispatch's column-major
// scales), counts [E] int32 valid rows -> d [E, slots, n] bf16; rows at or beyond counts[e] are left
// unwritten (unspecified).
torch::Tensor masked_grouped_gemm_fp8(const torch::Tensor& a, const torch::Tensor& sa, const torch::Tensor& counts,
                                      const torch::Tensor& b, const torch::Tensor& sb, int num_sms, double timeout_s) {
    TORCH_CHECK(a.is_cuda() && a.dim() == 3 && a.is_contiguous() && a.scalar_type() == torch::kFloat8_e4m3fn,
                "a must be a contiguous [E, slots, k] e4m3 tensor");
    TORCH_CHECK(b.dim() == 3 && b.is_contiguous() && b.scalar_type() == torch::kFloat8_e4m3fn, "b must be [E, n, k] e4m3");
    const int E = (int)a.size(0), slots = (int)a.size(1), k = (int)a.size(2), n = (int)b.size(1);
    TORCH_CHECK(b.size(0) == E && b.size(2) == k && k % 128 == 0 && n % 128 == 0, "k and n must be multiples of 128");
    TORCH_CHECK(E <= kMaxLocalExperts, "too many experts");
    TORCH_CHECK(sa.scalar_type() == torch::kFloat32 && sa.dim() == 3 && sa.size(0) == E && sa.size(1) == slots &&
                sa.size(2) == k / 128, "sa must be [E, slots, k/128] fp32");
    TORCH_CHECK(sb.scalar_type() == torch::kFloat32 && sb.is_contiguous() && sb.size(0) == E && sb.size(1) == n / 128 &&
                sb.size(2) == k / 128, "sb must be [E, n/128, k/128] fp32");
    TORCH_CHECK(counts.scalar_type() == torch::kInt32 && counts.is_contiguous() && counts.numel() == E && counts.is_cuda());
    auto d = torch::empty({E, slots, n}, a.options().dtype(torch::kBFloat16));
    if (num_sms <= 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    }
    MaskedGemmArgs g{};
    g.a = a.data_ptr();
    g.sa = sa.data_ptr<float>();
    g.sa_e = sa.stride(0);
    g.sa_m = sa.stride(1);
    g.sa_k = sa.stride(2);
    g.b = b.data_ptr();
    g.sb = sb.data_ptr<float>();
    g.counts = counts.data_ptr<int>();
    g.d = d.data_ptr();
    g.num_experts = E;
    g.slots = slots;
    g.n = n;
    g.k = k;
    g.st = op_status(timeout_s);
    const int rc = launch_masked_gemm_fp8(g, num_sms, at::cuda::getCurrentCUDAStream());
    TORCH_CHECK(rc == 0, "masked_grouped_gemm_fp8 launch failed (code " + std::to_string(rc) + ")");
    return d;
}

// bf16 grouped GEMM, both operands K-major. mode 0: a [rows, k] grouped by `offsets` (128-aligned),
// b [E, n, k] -> d [rows, n]. mode 1: a [m, Ktot], b [n, Ktot], offsets [E+1] over K -> d [E, m, n].
torch::Tensor grouped_gemm_bf16(const torch::Tensor& a, const torch::Tensor& b, const torch::Tensor& offsets,
                                const std::optional<torch::Tensor>& counts, int mode, int num_sms, double timeout_s,
                                bool a_mn_major, bool b_mn_major) {
    TORCH_CHECK(a.is_cuda() && a.dim() == 2 && a.is_contiguous() && a.scalar_type() == torch::kBFloat16);
    TORCH_CHECK(b.is_cuda() && b.is_contiguous() && b.scalar_type() == torch::kBFloat16);
    TORCH_CHECK(offsets.scalar_type() == torch::kInt32 && offsets.is_contiguous() && offsets.dim() == 1);
    TORCH_CHECK(mode == 0 || mode == 1, "mode must be 0 (M-grouped) or 1 (K-grouped)");
    const int E = (int)offsets.numel() - 1;
    TORCH_CHECK(E >= 1 && E <= 1024);
    Bf16GemmArgs g{};
    torch::Tensor d;
    if (mode == 0) {
        TORCH_CHECK(!a_mn_major, "mode 0: a is always [rows, k]");
        if (b_mn_major) {
            TORCH_CHECK(b.dim() == 3 && b.size(0) == E && b.size(1) == a.size(1), "mode 0, MN-major b: b must be [E, k, n]");
        } else {
            TORCH_CHECK(b.dim() == 3 && b.size(0) == E && b.size(2) == a.size(1), "mode 0: b must be [E, n, k]");
        }
        g.rows = (int)a.size(0);
        g.k = (int)a.size(1);
        g.n = (int)(b_mn_major ? b.size(2) : b.size(1));
        TORCH_CHECK(g.k % 64 == 0 && g.n % 128 == 0, "mode 0: k % 64 == 0 and n % 128 == 0");
        if (counts.has_value()) TORCH_CHECK(counts->scalar_type() == torch::kInt32 && counts->numel() == E);
        d = torch::empty({g.rows, g.n}, a.options());
    } else {
        g.m = (int)(a_mn_major ? a.size(1) : a.size(0));
        g.k = (int)(a_mn_major ? a.size(0) : a.size(1));
        TORCH_CHECK(b.dim() == 2 && (b_mn_major ? b.size(0) : b.size(1)) == g.k,
                    b_mn_major ? "mode 1, MN-major b: b must be [Ktot, n]" : "mode 1: b must be [n, Ktot]");
        g.n = (int)(b_mn_major ? b.size(1) : b.size(0));
        TORCH_CHECK(g.m % 128 == 0 && g.n % 128 == 0 && g.k % 64 == 0, "mode 1: m, n % 128 == 0 and Ktot % 64 == 0");
        d = torch::empty({E, g.m, g.n}, a.options());
    }
    if (num_sms <= 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    }
    g.a = a.data_ptr();
    g.b = b.data_ptr();
    g.offsets = offsets.data_ptr<int>();
    g.expert_counts = (mode == 0 && counts.has_value()) ? counts->data_ptr<int>() : nullptr;
    g.d = d.data_ptr();
    g.mode = mode;
    g.num_experts = E;
    g.a_mn_major = a_mn_major ? 1 : 0;
    g.b_mn_major = b_mn_major ? 1 : 0;
    g.st = op_status(timeout_s);
    const int rc = launch_grouped_gemm_bf16(g, num_sms, at::cuda::getCurrentCUDAStream());
    TORCH_CHECK(rc == 0, "grouped_gemm_bf16 launch failed (code " + std::to_string(rc) + ")");
    return d;
}

std::tuple<torch::Tensor, torch::Tensor> per_token_cast_to_fp8(const torch::Tensor& x, bool round_scale) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous() && x.scalar_type() == torch::kBFloat16,
                "x must be a contiguous CUDA bf16 [tokens, hidden] tensor");
    const int N = (int)x.size(0), H = (int)x.size(1);
    TORCH_CHECK(H % 128 == 0, "hidden must be a multiple of 128");
    auto out = torch::empty({N, H}, x.options().dtype(torch::kFloat8_e4m3fn));
    auto scales = torch::empty({N, H / 128}, x.options().dtype(torch::kFloat32));
    launch_per_token_cast_to_fp8(x.data_ptr(), N, H, out.data_ptr(), scales.data_ptr<float>(), round_scale ? 1 : 0,
                                 at::cuda::getCurrentCUDAStream());
    return {out, scales};
}

torch::Tensor per_token_cast_back(const torch::Tensor& x, const torch::Tensor& scales) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous() && x.scalar_type() == torch::kFloat8_e4m3fn);
    const int N = (int)x.size(0), H = (int)x.size(1);
    TORCH_CHECK(H % 128 == 0 && scales.scalar_type() == torch::kFloat32 && scales.size(0) == N && scales.size(1) == H / 128);
    auto s = scales.contiguous();
    auto out = torch::empty({N, H}, x.options().dtype(torch::kBFloat16));
    launch_per_token_cast_back(x.data_ptr(), s.data_ptr<float>(), N, H, out.data_ptr(), at::cuda::getCurrentCUDAStream());
    return out;
}

// a = silu(h[:, :I]) * h[:, I:] (bf16) and its 1x128 FP8 quantization.
// Expert weights [E, n, k] bf16 -> (fp8 e4m3 [E, n, k], fp32 128x128 block scales [E, n/128, k/128]).
std::tuple<torch::Tensor, torch::Tensor> quantize_weights_fp8(const torch::Tensor& w, bool round_scale) {
    TORCH_CHECK(w.is_cuda() && w.dim() == 3 && w.scalar_type() == torch::kBFloat16 && w.is_contiguous(),
                "quantize_weights_fp8: contiguous [E, n, k] bf16 CUDA tensor");
    const int E = (int)w.size(0), n = (int)w.size(1), k = (int)w.size(2);
    TORCH_CHECK(n % 128 == 0 && k % 128 == 0, "n and k must be multiples of 128");
    auto q = torch::empty({E, n, k}, w.options().dtype(torch::kFloat8_e4m3fn));
    auto s = torch::empty({E, n / 128, k / 128}, w.options().dtype(torch::kFloat32));
    launch_quantize_weights_fp8(w.data_ptr(), E, n, k, q.data_ptr(), s.data_ptr<float>(), at::cuda::getCurrentCUDAStream(),
                                round_scale ? 1 : 0);
    return {q, s};
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> swiglu_quant(const torch::Tensor& h, bool round_scale,
                                                                     const std::optional<torch::Tensor>& counts) {
    TORCH_CHECK(h.is_cuda() && h.is_contiguous() && h.scalar_type() == torch::kBFloat16);
    TORCH_CHECK(counts.has_value() ? h.dim() == 3 : h.dim() == 2, "h must be [rows, 2I], or [E, slots, 2I] with counts");
    const int inter = (int)h.size(-1) / 2;
    TORCH_CHECK(h.size(-1) % 256 == 0, "2*intermediate must be a multiple of 256");
    std::vector<int64_t> lead(h.sizes().begin(), h.sizes().end() - 1);
    const int rows = (int)(h.numel() / h.size(-1));
    auto shape = [&](int64_t last) {
        auto v = lead;
        v.push_back(last);
        return v;
    };
    const int* cnt = nullptr;
    int slots = 0;
    if (counts.has_value()) {
        TORCH_CHECK(counts->is_cuda() && counts->scalar_type() == torch::kInt32 && counts->is_contiguous() &&
                    counts->numel() == h.size(0), "counts must be int32 [E]");
        cnt = counts->data_ptr<int>();
        slots = (int)h.size(1);
    }
    auto a = torch::empty(shape(inter), h.options());
    auto aq = torch::empty(shape(inter), h.options().dtype(torch::kFloat8_e4m3fn));
    auto as = torch::empty(shape(inter / 128), h.options().dtype(torch::kFloat32));
    launch_swiglu_quant(h.data_ptr(), rows, inter, a.data_ptr(), aq.data_ptr(), as.data_ptr<float>(), round_scale ? 1 : 0,
                        at::cuda::getCurrentCUDAStream(), cnt, slots);
    return {a, aq, as};
}

// Grouped-by-expert permutation of dispatched tokens. Output rows are allocated for the worst case
// (`num_out_rows`, default N*K + E*(alignment-1)); rows past expert_offsets[E] are unused.
std::tuple<torch::Tensor, std::optional<torch::Tensor>, std::optional<torch::Tensor>, torch::Tensor, torch::Tensor, torch::Tensor>
permute(const torch::Tensor& x, const std::optional<torch::Tensor>& x_scales, const torch::Tensor& topk_idx,
        const std::optional<torch::Tensor>& probs, int num_experts, int alignment, int64_t num_out_rows, bool zero_padding) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous());
    TORCH_CHECK(x.scalar_type() == torch::kBFloat16 || x.scalar_type() == torch::kFloat8_e4m3fn);
    TORCH_CHECK(topk_idx.scalar_type() == torch::kInt64 && topk_idx.is_contiguous() && topk_idx.size(0) == x.size(0));
    TORCH_CHECK(num_experts > 0 && num_experts <= 4096 && alignment >= 1);
    const int N = (int)x.size(0), H = (int)x.size(1), K = (int)topk_idx.size(1);
    TORCH_CHECK((H * x.element_size()) % 16 == 0, "row bytes must be a multiple of 16");
    if (num_out_rows <= 0) num_out_rows = (int64_t)N * K + (int64_t)num_experts * (alignment - 1);
    auto i32 = x.options().dtype(torch::kInt32);
    const int chunks = (N + 31) / 32;
    auto counts = torch::empty({std::max(chunks, 1), num_experts}, i32);
    auto bases = torch::empty({std::max(chunks, 1), num_experts}, i32);
    auto offsets = torch::empty({num_experts + 1}, i32);
    auto ecounts = torch::empty({num_experts}, i32);
    auto row_map = torch::empty({N, K}, i32);
    auto x_perm = torch::empty({num_out_rows, H}, x.options());
    std::optional<torch::Tensor> sp, pp;
    PermuteArgs a{};
    if (x_scales.has_value()) {
        TORCH_CHECK(x_scales->scalar_type() == torch::kFloat32 && x_scales->is_contiguous() && x_scales->size(1) == H / 128);
        sp = torch::empty({num_out_rows, H / 128}, x.options().dtype(torch::kFloat32));
        a.x_scales = x_scales->data_ptr<float>();
        a.scales_perm = sp->data_ptr<float>();
    }
    if (probs.has_value()) {
        TORCH_CHECK(probs->scalar_type() == torch::kFloat32 && probs->is_contiguous() && probs->size(1) == K);
        pp = torch::zeros({num_out_rows}, x.options().dtype(torch::kFloat32));
        a.probs = probs->data_ptr<float>();
        a.probs_perm = pp->data_ptr<float>();
    }
    a.x = x.data_ptr();
    a.x_elem_bytes = (int)x.element_size();
    a.topk_idx = topk_idx.data_ptr<int64_t>();
    a.num_tokens = N;
    a.hidden = H;
    a.num_topk = K;
    a.num_experts = num_experts;
    a.alignment = alignment;
    a.counts = counts.data_ptr<int>();
    a.bases = bases.data_ptr<int>();
    a.expert_offsets = offsets.data_ptr<int>();
    a.expert_counts = ecounts.data_ptr<int>();
    a.row_map = row_map.data_ptr<int>();
    a.x_perm = x_perm.data_ptr();
    a.zero_padding = zero_padding ? 1 : 0;
    C10_CUDA_CHECK(launch_permute(a, at::cuda::getCurrentCUDAStream()));
    return {x_perm, sp, pp, row_map, offsets, ecounts};
}

torch::Tensor unpermute(const torch::Tensor& y, const torch::Tensor& row_map, const std::optional<torch::Tensor>& weights) {
    TORCH_CHECK(y.is_cuda() && y.dim() == 2 && y.is_contiguous() && y.scalar_type() == torch::kBFloat16);
    TORCH_CHECK(row_map.scalar_type() == torch::kInt32 && row_map.is_contiguous());
    const int N = (int)row_map.size(0), K = (int)row_map.size(1), H = (int)y.size(1);
    TORCH_CHECK(H % 8 == 0 && K <= kMaxTopk);
    if (weights.has_value())
        TORCH_CHECK(weights->scalar_type() == torch::kFloat32 && weights->is_contiguous() && weights->size(0) == N && weights->size(1) == K);
    auto out = torch::empty({N, H}, y.options());
    launch_unpermute(y.data_ptr(), row_map.data_ptr<int>(), weights.has_value() ? weights->data_ptr<float>() : nullptr, N, H, K,
                     out.data_ptr(), at::cuda::getCurrentCUDAStream());
    return out;
}

// MoE backward: g_y (caller-zeroed, [rows, H] bf16) receives bf16(g_tok[j] * w[j][k]) at row_map[j][k];
// returns g_w [N, K] fp32 = <g_tok[j], y[row_map[j][k]]> (0 where row_map is -1).
torch::Tensor unpermute_backward(const torch::Tensor& g_tok, const torch::Tensor& row_map, const torch::Tensor& w,
                                 const torch::Tensor& y, torch::Tensor& g_y) {
    TORCH_CHECK(g_tok.is_cuda() && g_tok.dim() == 2 && g_tok.is_contiguous() && g_tok.scalar_type() == torch::kBFloat16);
    TORCH_CHECK(row_map.scalar_type() == torch::kInt32 && row_map.is_contiguous() && row_map.dim() == 2);
    const int N = (int)row_map.size(0), K = (int)row_map.size(1), H = (int)g_tok.size(1);
    TORCH_CHECK(g_tok.size(0) >= N, "g_tok must cover every row of row_map");
    TORCH_CHECK(K <= kMaxTopk && H % 8 == 0, "top-k <= 16 and hidden % 8 == 0");
    TORCH_CHECK(w.scalar_type() == torch::kFloat32 && w.is_contiguous() && w.size(0) == N && w.size(1) == K);
    for (const torch::Tensor* t : {&y, static_cast<const torch::Tensor*>(&g_y)})
        TORCH_CHECK(t->is_cuda() && t->dim() == 2 && t->is_contiguous() && t->scalar_type() == torch::kBFloat16 && t->size(1) == H);
    TORCH_CHECK(g_y.size(0) == y.size(0), "g_y and y have the same rows");
    auto g_w = torch::empty({N, K}, w.options());
    launch_unpermute_backward(g_tok.data_ptr(), row_map.data_ptr<int>(), w.data_ptr<float>(), y.data_ptr(), N, H, K,
                              (int)y.size(0), g_y.data_ptr(), g_w.data_ptr<float>(), op_status(10.0),
                              at::cuda::getCurrentCUDAStream());
    return g_w;
}

torch::Tensor swiglu_backward(const torch::Tensor& h, const torch::Tensor& g_a) {
    TORCH_CHECK(h.is_cuda() && h.dim() == 2 && h.is_contiguous() && h.scalar_type() == torch::kBFloat16);
    const int64_t rows = h.size(0);
    const int inter = (int)h.size(1) / 2;
    TORCH_CHECK(h.size(1) % 16 == 0, "2*intermediate must be a multiple of 16");
    TORCH_CHECK(g_a.is_contiguous() && g_a.scalar_type() == torch::kBFloat16 && g_a.dim() == 2 && g_a.size(0) == rows &&
                g_a.size(1) == inter);
    auto g_h = torch::empty_like(h);
    launch_swiglu_backward(h.data_ptr(), g_a.data_ptr(), rows, inter, g_h.data_ptr(), at::cuda::getCurrentCUDAStream());
    return g_h;
}

void zero_group_padding(const std::vector<torch::Tensor>& tensors, const torch::Tensor& offsets, const torch::Tensor& counts) {
    TORCH_CHECK(tensors.size() <= 3, "at most three tensors per call");
    TORCH_CHECK(offsets.scalar_type() == torch::kInt32 && counts.scalar_type() == torch::kInt32 && offsets.is_contiguous() &&
                counts.is_contiguous() && offsets.numel() == counts.numel() + 1);
    ZeroPaddingArgs a{};
    for (size_t i = 0; i < tensors.size(); ++i) {
        const auto& t = tensors[i];
        TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.is_contiguous(), "grouped tensors must be contiguous 2D CUDA tensors");
        a.ptr[i] = t.data_ptr();
        a.row_bytes[i] = t.size(1) * t.element_size();
        TORCH_CHECK(a.row_bytes[i] % 16 == 0, "row bytes must be a multiple of 16");
    }
    a.num_tensors = (int)tensors.size();
    a.offsets = offsets.data_ptr<int>();
    a.counts = counts.data_ptr<int>();
    launch_zero_group_padding(a, (int)counts.numel(), at::cuda::getCurrentCUDAStream());
}

// Engram rows from storage that lies at caller-given device addresses, one per rank (the elastic
// API's hybrid mode: host segments registered with CUDA): out[t] = row (idx % entries_per_rank) of
// rank idx / entries_per_rank; a bad index gives a zero row and reports kErrBounds. Same kernel as
// the symmetric region's fetch.
torch::Tensor engram_fetch_rows(const torch::Tensor& indices, const std::vector<int64_t>& bases, int64_t entries_per_rank,
                                int64_t hidden, int num_sms, double timeout_s) {
    TORCH_CHECK(indices.is_cuda() && indices.is_contiguous() && indices.dim() == 1 && indices.scalar_type() == torch::kInt32,
                "engram indices: contiguous [num_tokens] int32 CUDA tensor");
    TORCH_CHECK(!bases.empty() && (int)bases.size() <= kMaxRanks, "one storage address per rank (1..8)");
    TORCH_CHECK(entries_per_rank > 0 && entries_per_rank * (int64_t)bases.size() < ((int64_t)1 << 31), "entries per rank");
    TORCH_CHECK(hidden > 0 && (hidden * 2) % 16 == 0, "engram hidden * 2 bytes must be a multiple of 16");
    for (int64_t b : bases) TORCH_CHECK(b != 0 && b % 16 == 0, "storage addresses must be 16-byte aligned");
    auto out = torch::empty({indices.size(0), hidden}, indices.options().dtype(torch::kBFloat16));
    EngramFetchArgs a{};
    for (size_t r = 0; r < bases.size(); ++r) a.storage.base[r] = reinterpret_cast<void*>(bases[r]);
    a.indices = indices.data_ptr<int>();
    a.out = static_cast<uint8_t*>(out.data_ptr());
    a.num_tokens = (int)indices.size(0);
    a.entries_per_rank = (int)entries_per_rank;
    a.row_bytes = (int)(hidden * 2);
    a.num_ranks = (int)bases.size();
    a.st = op_status(timeout_s);
    if (num_sms <= 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    }
    launch_engram_fetch(a, num_sms, at::cuda::getCurrentCUDAStream());
    TORCH_CHECK(cudaGetLastError() == cudaSuccess, "engram_fetch_rows launch failed");
    return out;
}

}  // namespace

void register_ops(pybind11::module_& m) {
    m.def("engram_fetch_rows", &engram_fetch_rows, pybind11::arg("indices"), pybind11::arg("bases"),
          pybind11::arg("entries_per_rank"), pybind11::arg("hidden"), pybind11::arg("num_sms") = 0,
          pybind11::arg("timeout_s") = 10.0);
    m.def("unpermute_backward", &unpermute_backward);
    m.def("swiglu_backward", &swiglu_backward);
    m.def("zero_group_padding", &zero_group_padding);
    m.def("permute", &permute, pybind11::arg("x"), pybind11::arg("x_scales"), pybind11::arg("topk_idx"), pybind11::arg("probs"),
          pybind11::arg("num_experts"), pybind11::arg("alignment") = 1, pybind11::arg("num_out_rows") = 0,
          pybind11::arg("zero_padding") = false);
    m.def("unpermute", &unpermute);
    m.def("swiglu_quant", &swiglu_quant, pybind11::arg("h"), pybind11::arg("round_scale") = false,
          pybind11::arg("counts") = std::nullopt);
    m.def("quantize_weights_fp8", &quantize_weights_fp8, pybind11::arg("w"), pybind11::arg("round_scale") = false);
    m.def("grouped_gemm_bf16", &grouped_gemm_bf16, pybind11::arg("a"), pybind11::arg("b"), pybind11::arg("offsets"),
          pybind11::arg("counts") = std::nullopt, pybind11::arg("mode") = 0, pybind11::arg("num_sms") = 0,
          pybind11::arg("timeout_s") = 10.0, pybind11::arg("a_mn_major") = false, pybind11::arg("b_mn_major") = false);
    m.def("masked_grouped_gemm_fp8", &masked_grouped_gemm_fp8, pybind11::arg("a"), pybind11::arg("sa"),
          pybind11::arg("counts"), pybind11::arg("b"), pybind11::arg("sb"), pybind11::arg("num_sms") = 0,
          pybind11::arg("timeout_s") = 100.0);
    m.def("grouped_gemm_fp8", &grouped_gemm_fp8, pybind11::arg("a"), pybind11::arg("sa"), pybind11::arg("b"), pybind11::arg("sb"),
          pybind11::arg("offsets"), pybind11::arg("counts") = pybind11::none(), pybind11::arg("num_sms") = 0,
          pybind11::arg("timeout_s") = 10.0, pybind11::arg("ue8m0") = false);
    m.def("op_error_state", &op_error_state, pybind11::arg("clear") = false);
    m.def("per_token_cast_to_fp8", &per_token_cast_to_fp8, pybind11::arg("x"), pybind11::arg("round_scale") = false);
    m.def("per_token_cast_back", &per_token_cast_back);
}

}  // namespace ep
