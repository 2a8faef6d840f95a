// PyTorch operators over the C ABI: torch.ops.gdn.chunk_fwd and torch.ops.gdn.decode_step.
//
// The reference's hot path is a Python function (fast_chunk_gated_delta_rule,
// qwen3_5_cutedsl_kernels.py:462-567); this package keeps that signature in a
// thin Python shim (ops.py) and puts the per-call work of a drop-in op here,
// in C++: argument checks, output and workspace allocation through PyTorch's
// caching allocator, the strided tensor descriptors and the call into
// libgdn_b200.so on the current CUDA stream.  Registered for the CUDA dispatch
// key (and for CPU, where it raises: there is no CPU path), so the ops also
// work inside torch.compile graphs and CUDA-graph capture (no host
// synchronisation on the call path once a device has been used).
//
//   gdn::chunk_fwd(query, key, value, g, beta, chunk_size=64, initial_state=None,
//                  output_final_state=False, use_qk_l2norm_in_kernel=False,
//                  workspace=None) -> (out, final_state)
//     = fast_chunk_gated_delta_rule (qwen3_5_cutedsl_kernels.py:462-473);
//       final_state is None unless output_final_state.
//   gdn::decode_step(query, key, value, g, beta, initial_state, output_final_state,
//                    use_qk_l2norm_in_kernel=False, out_state=None) -> (out, final_state)
//     = torch_recurrent_gated_delta_rule (qwen3_5_transformers.py:190-229);
//       out_state (fp32 [B,H,Dk,Dv], may be initial_state) receives the state in place.
//
// Errors raise RuntimeError whose message starts with the gdn_status name, as the
// Python shim's GDNError does; a failure a kernel reported in the device error word
// surfaces as GDN_ERR_KERNEL at the next op on that device.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <algorithm>
#include <cstdio>
#include <tuple>

#include "gdn_b200.h"

namespace {

int dtype_code(at::ScalarType t) {
    switch (t) {
        case at::kFloat: return GDN_F32;
        case at::kBFloat16: return GDN_BF16;
        case at::kHalf: return GDN_F16;
        default: return -1;
    }
}

gdn_tensor desc(const at::Tensor& t) {
    gdn_tensor d{};
    d.data = t.numel() > 0 ? t.data_ptr() : nullptr;
    d.dtype = dtype_code(t.scalar_type());
    d.ndim = (int32_t)t.dim();
    for (int i = 0; i < 4; ++i) {
        d.shape[i] = i < t.dim() ? t.size(i) : 1;
        d.stride[i] = i < t.dim() ? t.stride(i) : 1;
    }
    return d;
}

// A kernel operand: `ndim` dims on `dev`, a float dtype the kernels read (others become fp32), a contiguous
// head dimension.
at::Tensor operand(const at::Tensor& x, const char* name, int64_t ndim, const c10::Device& dev) {
    TORCH_CHECK(x.dim() == ndim, name, " must have ", ndim, " dims, got shape ", x.sizes());
    TORCH_CHECK(x.is_cuda(), name, " is on ", x.device(), "; the GatedDeltaNet kernels need CUDA tensors (no CPU path)");
    TORCH_CHECK(x.device() == dev, name, " is on ", x.device(), ", query on ", dev);
    at::Tensor y = dtype_code(x.scalar_type()) < 0 ? x.to(at::kFloat) : x;
    if (ndim == 4 && y.size(-1) > 1 && y.stride(-1) != 1) y = y.contiguous();
    return y;
}

c10::optional<at::Tensor> state_in(const c10::optional<at::Tensor>& s, int64_t B, int64_t H, int64_t Dk, int64_t Dv,
                                   const c10::Device& dev) {
    if (!s.has_value() || !s->defined()) return c10::nullopt;
    TORCH_CHECK(s->dim() == 4 && s->size(0) == B && s->size(1) == H && s->size(2) == Dk && s->size(3) == Dv,
                "initial_state must have shape [", B, ", ", H, ", ", Dk, ", ", Dv, "], got ", s->sizes());
    TORCH_CHECK(s->device() == dev, "initial_state is on ", s->device(), ", expected ", dev);
    return s->to(at::kFloat).contiguous();
}

void check(int rc) { TORCH_CHECK(rc == GDN_OK, gdn_status_name(rc), ": ", gdn_last_error()); }

// A failure an earlier kernel on the current device reported (host mirror of the device error word: no
// synchronisation unless a bit is set).
void raise_pending(const c10::Device& dev) {
    unsigned int bits = gdn_device_error_pending();
    if (!bits) return;
    const unsigned int all = gdn_device_error(1);
    if (all) bits = all;
    char hex[16];
    std::snprintf(hex, sizeof(hex), "0x%x", bits);
    TORCH_CHECK(false, "GDN_ERR_KERNEL: a kernel on ", dev, " reported device error bits ", hex,
                "; the outputs of the call that launched it are not valid");
}

std::tuple<at::Tensor, at::Tensor> chunk_fwd(const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
                                             const at::Tensor& g, const at::Tensor& beta, int64_t chunk_size,
                                             const c10::optional<at::Tensor>& initial_state, bool output_final_state,
                                             bool use_qk_l2norm_in_kernel, const c10::optional<at::Tensor>& workspace) {
    TORCH_CHECK(query.is_cuda(), "query is on ", query.device(),
                "; the GatedDeltaNet kernels need CUDA tensors (no CPU path)");
    const c10::Device dev = query.device();
    c10::cuda::CUDAGuard guard(dev);
    at::Tensor q = operand(query, "query", 4, dev), k = operand(key, "key", 4, dev);
    at::Tensor v = operand(value, "value", 4, dev);
    at::Tensor gg = operand(g, "g", 3, dev), bb = operand(beta, "beta", 3, dev);
    const int64_t B = q.size(0), T = q.size(1), H = q.size(2), Dk = q.size(3), Dv = v.size(3);
    auto h0 = state_in(initial_state, B, H, Dk, Dv, dev);
    at::Tensor out = at::empty({B, T, H, Dv}, q.options());
    at::Tensor fin = output_final_state ? at::empty({B, H, Dk, Dv}, q.options().dtype(at::kFloat)) : at::Tensor();
    raise_pending(dev);
    const size_t need = gdn_chunk_workspace_bytes(B, T, H, Dk, Dv, dtype_code(q.scalar_type()));
    at::Tensor ws;
    if (workspace.has_value() && workspace->defined()) {
        TORCH_CHECK(workspace->device() == dev, "workspace is on ", workspace->device(), "; it must be a CUDA tensor on ",
                    dev);
        if (workspace->is_contiguous() && (size_t)workspace->nbytes() >= need) ws = *workspace;
    }
    if (!ws.defined()) ws = at::empty({(int64_t)std::max<size_t>(need, 1)}, q.options().dtype(at::kByte));
    gdn_tensor dq = desc(q), dk = desc(k), dv = desc(v), dg = desc(gg), db = desc(bb), dout = desc(out);
    check(gdn_chunk_gated_delta_rule(&dq, &dk, &dv, &dg, &db, (int)chunk_size, h0 ? h0->data_ptr<float>() : nullptr,
                                     output_final_state ? 1 : 0, use_qk_l2norm_in_kernel ? 1 : 0, &dout,
                                     fin.defined() ? fin.data_ptr<float>() : nullptr, ws.data_ptr(), ws.nbytes(),
                                     at::cuda::getCurrentCUDAStream(dev.index()).stream()));
    if (out.scalar_type() != query.scalar_type()) out = out.to(query.scalar_type());
    return {out, fin};
}

std::tuple<at::Tensor, at::Tensor> decode_step(const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
                                               const at::Tensor& g, const at::Tensor& beta,
                                               const c10::optional<at::Tensor>& initial_state, bool output_final_state,
                                               bool use_qk_l2norm_in_kernel, const c10::optional<at::Tensor>& out_state) {
    TORCH_CHECK(query.is_cuda(), "query is on ", query.device(),
                "; the GatedDeltaNet kernels need CUDA tensors (no CPU path)");
    const c10::Device dev = query.device();
    c10::cuda::CUDAGuard guard(dev);
    at::Tensor q = operand(query, "query", 4, dev), k = operand(key, "key", 4, dev);
    at::Tensor v = operand(value, "value", 4, dev);
    at::Tensor gg = operand(g, "g", 3, dev), bb = operand(beta, "beta", 3, dev);
    const int64_t B = q.size(0), T = q.size(1), H = q.size(2), Dk = q.size(3), Dv = v.size(3);
    auto h0 = state_in(initial_state, B, H, Dk, Dv, dev);
    at::Tensor out = at::empty({B, T, H, Dv}, q.options());
    at::Tensor fin;
    if (output_final_state) {
        if (out_state.has_value() && out_state->defined()) {
            const at::Tensor& s = *out_state;
            TORCH_CHECK(s.scalar_type() == at::kFloat && s.dim() == 4 && s.size(0) == B && s.size(1) == H &&
                            s.size(2) == Dk && s.size(3) == Dv && s.is_contiguous() && s.device() == dev,
                        "out_state must be a contiguous fp32 [B,H,Dk,Dv] tensor on the query's device");
            fin = s;
        } else {
            fin = at::empty({B, H, Dk, Dv}, q.options().dtype(at::kFloat));
        }
    }
    raise_pending(dev);
    gdn_tensor dq = desc(q), dk = desc(k), dv = desc(v), dg = desc(gg), db = desc(bb), dout = desc(out);
    check(gdn_recurrent_gated_delta_rule(&dq, &dk, &dv, &dg, &db, h0 ? h0->data_ptr<float>() : nullptr,
                                         output_final_state ? 1 : 0, use_qk_l2norm_in_kernel ? 1 : 0, &dout,
                                         fin.defined() ? fin.data_ptr<float>() : nullptr,
                                         at::cuda::getCurrentCUDAStream(dev.index()).stream()));
    if (out.scalar_type() != query.scalar_type()) out = out.to(query.scalar_type());
    return {out, fin};
}

}  // namespace

TORCH_LIBRARY(gdn, m) {
    m.def("chunk_fwd(Tensor query, Tensor key, Tensor value, Tensor g, Tensor beta, int chunk_size=64, "
          "Tensor? initial_state=None, bool output_final_state=False, bool use_qk_l2norm_in_kernel=False, "
          "Tensor? workspace=None) -> (Tensor, Tensor)");
    m.def("decode_step(Tensor query, Tensor key, Tensor value, Tensor g, Tensor beta, Tensor? initial_state, "
          "bool output_final_state, bool use_qk_l2norm_in_kernel=False, Tensor(a!)? out_state=None) -> "
          "(Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(gdn, CUDA, m) {
    m.impl("chunk_fwd", &chunk_fwd);
    m.impl("decode_step", &decode_step);
}

TORCH_LIBRARY_IMPL(gdn, CPU, m) {  // raises "... need CUDA tensors (no CPU path)"
    m.impl("chunk_fwd", &chunk_fwd);
    m.impl("decode_step", &decode_step);
}
