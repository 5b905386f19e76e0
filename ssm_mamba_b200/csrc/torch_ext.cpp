// Thin torch binding of the C ABI (include/ssm_b200.h): checks tensors, allocates outputs
// with the caching allocator, fills the argument structs and calls the library on the
// current stream.  The checks follow the reference host glue (nmquan1503/ssm-mamba,
// csrc/selective_scan/selective_scan.cpp:15-32, 229-268, 314-351) and raise the same kind
// of RuntimeError; there is no CPU path -- non-CUDA tensors are rejected.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <optional>
#include <vector>

#include "../../include/ssm_b200.h"

namespace {

int32_t dtype_code(const at::Tensor& t) {
    if (t.scalar_type() == at::kFloat) return SSM_F32;
    if (t.scalar_type() == at::kBFloat16) return SSM_BF16;
    TORCH_CHECK(false, "selective scan tensors must be float32 or bfloat16, got ", t.scalar_type());
    return -1;
}

void check_cuda(const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

// (batch, dim, seqlen) with unit innermost stride
void check_bdl(const at::Tensor& t, const char* name, int64_t B, int64_t D, int64_t L, at::ScalarType st) {
    check_cuda(t, name);
    TORCH_CHECK(t.dim() == 3, name, " must be a 3D tensor");
    TORCH_CHECK(t.size(0) == B && t.size(1) == D && t.size(2) == L, name, " must have shape (", B, ", ", D,
                ", ", L, ")");
    TORCH_CHECK(t.scalar_type() == st, name, " must have dtype ", st);
    TORCH_CHECK(t.stride(2) == 1, name, " must be contiguous along the sequence");
}

void check_f32(const at::Tensor& t, const char* name, std::vector<int64_t> shape) {
    check_cuda(t, name);
    TORCH_CHECK(t.scalar_type() == at::kFloat, name, " must be float32 tensor");
    TORCH_CHECK(t.sizes() == at::IntArrayRef(shape), name, " has the wrong shape");
}

void ok(int rc) {
    if (rc != SSM_OK) TORCH_CHECK(false, ssm_last_error());
}

template <typename T>
T* ptr(const std::optional<at::Tensor>& t) {
    return t.has_value() ? static_cast<T*>(t->data_ptr()) : nullptr;
}

struct Common {
    int64_t B, D, L, N;
    int32_t dt;
};

Common check_inputs(const at::Tensor& u, const at::Tensor& delta, const at::Tensor& A, const at::Tensor& Bm,
                    const at::Tensor& Cm, const std::optional<at::Tensor>& D, const std::optional<at::Tensor>& z,
                    const std::optional<at::Tensor>& delta_bias, const std::optional<at::Tensor>& h_init,
                    const std::optional<at::Tensor>& length) {
    check_cuda(u, "u");
    TORCH_CHECK(u.dim() == 3, "u must be a 3D tensor");
    Common c{u.size(0), u.size(1), u.size(2), 0, dtype_code(u)};
    TORCH_CHECK(A.dim() == 2, "A must be a 2D tensor");
    c.N = A.size(1);
    TORCH_CHECK(c.N <= 256, "selective_scan only supports state_dim <= 256");
    check_bdl(u, "u", c.B, c.D, c.L, u.scalar_type());
    check_bdl(delta, "delta", c.B, c.D, c.L, u.scalar_type());
    check_cuda(A, "A");
    TORCH_CHECK(A.scalar_type() == at::kFloat && A.size(0) == c.D && A.stride(1) == 1,
                "A must be float32 of shape (dim, state_dim) with unit state stride");
    for (auto* bc : {&Bm, &Cm}) {
        const char* nm = bc == &Bm ? "B" : "C";
        check_cuda(*bc, nm);
        TORCH_CHECK(bc->dim() == 3 && bc->size(0) == c.B && bc->size(1) == c.N && bc->size(2) == c.L, nm,
                    " must have shape (batch, state_dim, seq_len)");
        TORCH_CHECK(bc->scalar_type() == u.scalar_type(), nm, " must have the dtype of u");
        TORCH_CHECK(bc->stride(2) == 1, nm, " must be contiguous along the sequence");
    }
    if (D) check_f32(*D, "D", {c.D});
    if (D) TORCH_CHECK(D->is_contiguous(), "D must be contiguous");
    if (delta_bias) check_f32(*delta_bias, "delta_bias", {c.D});
    if (delta_bias) TORCH_CHECK(delta_bias->is_contiguous(), "delta_bias must be contiguous");
    if (z) check_bdl(*z, "z", c.B, c.D, c.L, u.scalar_type());
    if (h_init) {
        check_f32(*h_init, "h_init", {c.B, c.D, c.N});
        TORCH_CHECK(h_init->is_contiguous(), "h_init must be contiguous");
    }
    if (length) {
        TORCH_CHECK(length->is_cuda(), "length must be a CUDA tensor");
        TORCH_CHECK(length->scalar_type() == at::kLong, "length must be long tensor");
        TORCH_CHECK(length->is_contiguous(), "length must be contiguous");
        TORCH_CHECK(length->dim() == 1 && length->size(0) == c.B, "length must have shape (batch_size,)");
    }
    return c;
}

ssm_scan_fwd_args fwd_args(const Common& c, const at::Tensor& u, const at::Tensor& delta, const at::Tensor& A,
                           const at::Tensor& Bm, const at::Tensor& Cm, const std::optional<at::Tensor>& D,
                           const std::optional<at::Tensor>& z, const std::optional<at::Tensor>& delta_bias,
                           const std::optional<at::Tensor>& h_init, const std::optional<at::Tensor>& length,
                           bool padding_right, bool delta_softplus) {
    ssm_scan_fwd_args a;
    memset(&a, 0, sizeof(a));
    a.batch = c.B; a.dim = c.D; a.seqlen = c.L; a.dstate = c.N; a.dtype = c.dt;
    a.delta_softplus = delta_softplus; a.padding_right = padding_right;
    a.u = u.data_ptr(); a.u_batch_stride = u.stride(0); a.u_dim_stride = u.stride(1);
    a.delta = delta.data_ptr(); a.delta_batch_stride = delta.stride(0); a.delta_dim_stride = delta.stride(1);
    a.A = A.data_ptr<float>(); a.A_dim_stride = A.stride(0);
    a.B = Bm.data_ptr(); a.B_batch_stride = Bm.stride(0); a.B_state_stride = Bm.stride(1);
    a.C = Cm.data_ptr(); a.C_batch_stride = Cm.stride(0); a.C_state_stride = Cm.stride(1);
    a.D = ptr<const float>(D);
    if (z) { a.z = z->data_ptr(); a.z_batch_stride = z->stride(0); a.z_dim_stride = z->stride(1); }
    a.delta_bias = ptr<const float>(delta_bias);
    a.h_init = ptr<const float>(h_init);
    a.length = ptr<const int64_t>(length);
    return a;
}

// Forward into given out (and y) tensors, which may be strided views (unit innermost
// stride).  ckpt_mode: 0 none, 1 compact (for ssm_scan_bwd), 2 reference layout.
// Returns [out, y or undefined, ckpt or undefined, h_last or undefined].
std::vector<at::Tensor> scan_fwd_out(const at::Tensor& u, const at::Tensor& delta, const at::Tensor& A,
                                     const at::Tensor& Bm, const at::Tensor& Cm, const std::optional<at::Tensor>& D,
                                     const std::optional<at::Tensor>& z, const std::optional<at::Tensor>& delta_bias,
                                     const std::optional<at::Tensor>& h_init, const std::optional<at::Tensor>& length,
                                     bool padding_right, bool delta_softplus, const at::Tensor& out,
                                     const std::optional<at::Tensor>& y, int64_t ckpt_mode, bool want_h_last) {
    Common c = check_inputs(u, delta, A, Bm, Cm, D, z, delta_bias, h_init, length);
    c10::cuda::CUDAGuard guard(u.device());
    ssm_scan_fwd_args a = fwd_args(c, u, delta, A, Bm, Cm, D, z, delta_bias, h_init, length, padding_right,
                                   delta_softplus);
    check_bdl(out, "out", c.B, c.D, c.L, u.scalar_type());
    at::Tensor ck, hl;
    a.out = out.data_ptr(); a.out_batch_stride = out.stride(0); a.out_dim_stride = out.stride(1);
    if (y) {
        check_bdl(*y, "y", c.B, c.D, c.L, u.scalar_type());
        a.y = y->data_ptr(); a.y_batch_stride = y->stride(0); a.y_dim_stride = y->stride(1);
    }
    const auto f32 = u.options().dtype(at::kFloat);
    if (ckpt_mode == 1) {
        const int64_t k = ssm_scan_ckpt_len(c.N);
        ck = at::empty({c.B, ssm_scan_num_ckpt(c.L, k), c.D, c.N}, f32);
        a.ckpt = ck.data_ptr<float>(); a.ckpt_format = SSM_CKPT_COMPACT; a.ckpt_len = k;
    } else if (ckpt_mode == 2) {
        ck = at::empty({c.B, c.D, ssm_scan_num_ckpt(c.L, 128), 2 * c.N}, f32);
        a.ckpt = ck.data_ptr<float>(); a.ckpt_format = SSM_CKPT_REFERENCE; a.ckpt_len = 128;
    }
    if (want_h_last) {
        hl = at::empty({c.B, c.D, c.N}, f32);
        a.h_last = hl.data_ptr<float>();
    }
    ok(ssm_scan_fwd(&a, at::cuda::getCurrentCUDAStream().stream()));
    return {out, y ? *y : at::Tensor(), ck, hl};
}

std::vector<at::Tensor> scan_fwd(const at::Tensor& u, const at::Tensor& delta, const at::Tensor& A,
                                 const at::Tensor& Bm, const at::Tensor& Cm, const std::optional<at::Tensor>& D,
                                 const std::optional<at::Tensor>& z, const std::optional<at::Tensor>& delta_bias,
                                 const std::optional<at::Tensor>& h_init, const std::optional<at::Tensor>& length,
                                 bool padding_right, bool delta_softplus, bool want_y, int64_t ckpt_mode,
                                 bool want_h_last) {
    check_cuda(u, "u");
    TORCH_CHECK(u.dim() == 3, "u must be a 3D tensor");
    at::Tensor out = at::empty(u.sizes(), u.options());
    std::optional<at::Tensor> y;
    if (want_y) y = at::empty(u.sizes(), u.options());
    return scan_fwd_out(u, delta, A, Bm, Cm, D, z, delta_bias, h_init, length, padding_right, delta_softplus, out,
                        y, ckpt_mode, want_h_last);
}

// Compact checkpoints rebuilt from the reference-layout chunk states.
at::Tensor ckpt_from_reference(const at::Tensor& u, const at::Tensor& delta, const at::Tensor& A,
                               const at::Tensor& Bm, const at::Tensor& Cm,
                               const std::optional<at::Tensor>& delta_bias, const std::optional<at::Tensor>& h_init,
                               const std::optional<at::Tensor>& length, bool padding_right, bool delta_softplus,
                               const at::Tensor& ref_ckpt) {
    Common c = check_inputs(u, delta, A, Bm, Cm, std::nullopt, std::nullopt, delta_bias, h_init, length);
    c10::cuda::CUDAGuard guard(u.device());
    check_f32(ref_ckpt, "h", {c.B, c.D, ssm_scan_num_ckpt(c.L, 128), 2 * c.N});
    TORCH_CHECK(ref_ckpt.is_contiguous(), "h must be contiguous");
    ssm_scan_fwd_args a = fwd_args(c, u, delta, A, Bm, Cm, std::nullopt, std::nullopt, delta_bias, h_init, length,
                                   padding_right, delta_softplus);
    const int64_t k = ssm_scan_ckpt_len(c.N);
    at::Tensor ck = at::empty({c.B, ssm_scan_num_ckpt(c.L, k), c.D, c.N}, u.options().dtype(at::kFloat));
    a.ckpt = ck.data_ptr<float>(); a.ckpt_format = SSM_CKPT_COMPACT; a.ckpt_len = k;
    ok(ssm_scan_ckpt_from_reference(&a, ref_ckpt.data_ptr<float>(), at::cuda::getCurrentCUDAStream().stream()));
    return ck;
}

// Backward into given du, ddelta, dB, dC (and dz) tensors, which may be strided views
// (unit innermost stride).  Returns [du, ddelta, dA, dB, dC, dD?, ddelta_bias?, dz?, dh_init?].
std::vector<at::Tensor> scan_bwd_out(const at::Tensor& u, const at::Tensor& delta, const at::Tensor& A,
                                     const at::Tensor& Bm, const at::Tensor& Cm, const std::optional<at::Tensor>& D,
                                     const std::optional<at::Tensor>& z, const std::optional<at::Tensor>& delta_bias,
                                     const std::optional<at::Tensor>& h_init, const std::optional<at::Tensor>& length,
                                     bool padding_right, bool delta_softplus, const std::optional<at::Tensor>& y,
                                     const at::Tensor& ckpt, const at::Tensor& dout,
                                     const std::optional<at::Tensor>& dh_last, const at::Tensor& du,
                                     const at::Tensor& ddelta, const at::Tensor& dB, const at::Tensor& dC,
                                     const std::optional<at::Tensor>& dz_out) {
    Common c = check_inputs(u, delta, A, Bm, Cm, D, z, delta_bias, h_init, length);
    c10::cuda::CUDAGuard guard(u.device());
    check_bdl(dout, "dout", c.B, c.D, c.L, u.scalar_type());
    const int64_t k = ssm_scan_ckpt_len(c.N);
    check_f32(ckpt, "ckpt", {c.B, ssm_scan_num_ckpt(c.L, k), c.D, c.N});
    TORCH_CHECK(ckpt.is_contiguous(), "ckpt must be contiguous");
    if (z) {
        TORCH_CHECK(y.has_value(), "the pre-gate output y is needed when z is given");
        check_bdl(*y, "y", c.B, c.D, c.L, u.scalar_type());
    }
    if (dh_last) {
        check_f32(*dh_last, "dh_last", {c.B, c.D, c.N});
        TORCH_CHECK(dh_last->is_contiguous(), "dh_last must be contiguous");
    }
    ssm_scan_bwd_args a;
    memset(&a, 0, sizeof(a));
    a.batch = c.B; a.dim = c.D; a.seqlen = c.L; a.dstate = c.N; a.dtype = c.dt;
    a.delta_softplus = delta_softplus; a.padding_right = padding_right;
    a.reference_length_semantics = 1;
    a.u = u.data_ptr(); a.u_batch_stride = u.stride(0); a.u_dim_stride = u.stride(1);
    a.delta = delta.data_ptr(); a.delta_batch_stride = delta.stride(0); a.delta_dim_stride = delta.stride(1);
    a.A = A.data_ptr<float>(); a.A_dim_stride = A.stride(0);
    a.B = Bm.data_ptr(); a.B_batch_stride = Bm.stride(0); a.B_state_stride = Bm.stride(1);
    a.C = Cm.data_ptr(); a.C_batch_stride = Cm.stride(0); a.C_state_stride = Cm.stride(1);
    a.D = ptr<const float>(D);
    if (z) { a.z = z->data_ptr(); a.z_batch_stride = z->stride(0); a.z_dim_stride = z->stride(1); }
    if (y) { a.y = y->data_ptr(); a.y_batch_stride = y->stride(0); a.y_dim_stride = y->stride(1); }
    a.delta_bias = ptr<const float>(delta_bias);
    a.h_init = ptr<const float>(h_init);
    a.length = ptr<const int64_t>(length);
    a.ckpt = ckpt.data_ptr<float>(); a.ckpt_format = SSM_CKPT_COMPACT; a.ckpt_len = k;
    a.dout = dout.data_ptr(); a.dout_batch_stride = dout.stride(0); a.dout_dim_stride = dout.stride(1);
    a.dh_last = ptr<const float>(dh_last);
    check_bdl(du, "du", c.B, c.D, c.L, u.scalar_type());
    check_bdl(ddelta, "ddelta", c.B, c.D, c.L, u.scalar_type());
    for (auto* t : {&dB, &dC}) {
        check_cuda(*t, "dB/dC");
        TORCH_CHECK(t->dim() == 3 && t->size(0) == c.B && t->size(1) == c.N && t->size(2) == c.L &&
                        t->stride(2) == 1 && t->scalar_type() == u.scalar_type(),
                    "dB and dC must have shape (batch, state_dim, seq_len), unit sequence stride");
    }
    at::Tensor dA = at::empty({c.D, c.N}, A.options());
    const auto f32 = u.options().dtype(at::kFloat);
    at::Tensor dD = D ? at::empty({c.D}, f32) : at::Tensor();
    at::Tensor dbias = delta_bias ? at::empty({c.D}, f32) : at::Tensor();
    at::Tensor dz;
    if (z) {
        TORCH_CHECK(dz_out.has_value(), "dz is needed when z is given");
        dz = *dz_out;
        check_bdl(dz, "dz", c.B, c.D, c.L, u.scalar_type());
    }
    at::Tensor dh_init = h_init ? at::empty({c.B, c.D, c.N}, f32) : at::Tensor();
    a.du = du.data_ptr(); a.du_batch_stride = du.stride(0); a.du_dim_stride = du.stride(1);
    a.ddelta = ddelta.data_ptr(); a.ddelta_batch_stride = ddelta.stride(0); a.ddelta_dim_stride = ddelta.stride(1);
    if (z) { a.dz = dz.data_ptr(); a.dz_batch_stride = dz.stride(0); a.dz_dim_stride = dz.stride(1); }
    a.dA = dA.data_ptr<float>();
    a.dB = dB.data_ptr(); a.dC = dC.data_ptr();
    a.dB_batch_stride = dB.stride(0); a.dB_state_stride = dB.stride(1);
    a.dC_batch_stride = dC.stride(0); a.dC_state_stride = dC.stride(1);
    a.dD = D ? dD.data_ptr<float>() : nullptr;
    a.ddelta_bias = delta_bias ? dbias.data_ptr<float>() : nullptr;
    a.dh_init = h_init ? dh_init.data_ptr<float>() : nullptr;
    const size_t ws_bytes = ssm_scan_bwd_workspace_size(&a);
    TORCH_CHECK(ws_bytes > 0, ssm_last_error());
    at::Tensor ws = at::empty({(int64_t)ws_bytes}, u.options().dtype(at::kByte));
    ok(ssm_scan_bwd(&a, ws.data_ptr(), ws_bytes, at::cuda::getCurrentCUDAStream().stream()));
    return {du, ddelta, dA, dB, dC, dD, dbias, dz, dh_init};
}

std::vector<at::Tensor> scan_bwd(const at::Tensor& u, const at::Tensor& delta, const at::Tensor& A,
                                 const at::Tensor& Bm, const at::Tensor& Cm, const std::optional<at::Tensor>& D,
                                 const std::optional<at::Tensor>& z, const std::optional<at::Tensor>& delta_bias,
                                 const std::optional<at::Tensor>& h_init, const std::optional<at::Tensor>& length,
                                 bool padding_right, bool delta_softplus, const std::optional<at::Tensor>& y,
                                 const at::Tensor& ckpt, const at::Tensor& dout,
                                 const std::optional<at::Tensor>& dh_last) {
    check_cuda(u, "u");
    TORCH_CHECK(u.dim() == 3, "u must be a 3D tensor");
    at::Tensor du = at::empty(u.sizes(), u.options());
    at::Tensor ddelta = at::empty(u.sizes(), u.options());
    at::Tensor dB = at::empty(Bm.sizes(), u.options());
    at::Tensor dC = at::empty(Cm.sizes(), u.options());
    std::optional<at::Tensor> dz;
    if (z) dz = at::empty(u.sizes(), u.options());
    return scan_bwd_out(u, delta, A, Bm, Cm, D, z, delta_bias, h_init, length, padding_right, delta_softplus, y,
                        ckpt, dout, dh_last, du, ddelta, dB, dC, dz);
}

// Sequence slices: end state from a zero start and sum of delta of every row.
std::vector<at::Tensor> chunk_state_fwd(const at::Tensor& u, const at::Tensor& delta, const at::Tensor& A,
                                        const at::Tensor& Bm, const std::optional<at::Tensor>& delta_bias,
                                        bool delta_softplus) {
    Common c = check_inputs(u, delta, A, Bm, Bm, std::nullopt, std::nullopt, delta_bias, std::nullopt,
                            std::nullopt);
    c10::cuda::CUDAGuard guard(u.device());
    ssm_scan_fwd_args a = fwd_args(c, u, delta, A, Bm, Bm, std::nullopt, std::nullopt, delta_bias, std::nullopt,
                                   std::nullopt, true, delta_softplus);
    const auto f32 = u.options().dtype(at::kFloat);
    at::Tensor h_end = at::empty({c.B, c.D, c.N}, f32);
    at::Tensor dsum = at::empty({c.B, c.D}, f32);
    ok(ssm_scan_chunk_state_fwd(&a, h_end.data_ptr<float>(), dsum.data_ptr<float>(),
                                at::cuda::getCurrentCUDAStream().stream()));
    return {h_end, dsum};
}

// Sequence slices: gradient into the state before every row, from a zero incoming gradient.
at::Tensor chunk_state_bwd(const at::Tensor& delta, const at::Tensor& A, const at::Tensor& Cm,
                           const std::optional<at::Tensor>& z, const std::optional<at::Tensor>& delta_bias,
                           bool delta_softplus, const at::Tensor& dout) {
    Common c = check_inputs(delta, delta, A, Cm, Cm, std::nullopt, z, delta_bias, std::nullopt, std::nullopt);
    c10::cuda::CUDAGuard guard(delta.device());
    check_bdl(dout, "dout", c.B, c.D, c.L, delta.scalar_type());
    ssm_scan_bwd_args a;
    memset(&a, 0, sizeof(a));
    a.batch = c.B; a.dim = c.D; a.seqlen = c.L; a.dstate = c.N; a.dtype = c.dt;
    a.delta_softplus = delta_softplus;
    a.delta = delta.data_ptr(); a.delta_batch_stride = delta.stride(0); a.delta_dim_stride = delta.stride(1);
    a.A = A.data_ptr<float>(); a.A_dim_stride = A.stride(0);
    a.C = Cm.data_ptr(); a.C_batch_stride = Cm.stride(0); a.C_state_stride = Cm.stride(1);
    if (z) { a.z = z->data_ptr(); a.z_batch_stride = z->stride(0); a.z_dim_stride = z->stride(1); }
    a.delta_bias = ptr<const float>(delta_bias);
    a.dout = dout.data_ptr(); a.dout_batch_stride = dout.stride(0); a.dout_dim_stride = dout.stride(1);
    at::Tensor g = at::empty({c.B, c.D, c.N}, delta.options().dtype(at::kFloat));
    ok(ssm_scan_chunk_state_bwd(&a, g.data_ptr<float>(), at::cuda::getCurrentCUDAStream().stream()));
    return g;
}

// Sequence slices: fold per-slice carries.  carry (S, batch, dim, N) with any slice stride,
// delta_sum (S, batch, dim); start: (R, batch, dim, N) summed over R, or None.
at::Tensor carry_compose(const at::Tensor& A, const at::Tensor& carry, const at::Tensor& delta_sum,
                         const std::optional<at::Tensor>& start, bool reverse) {
    check_cuda(carry, "carry");
    TORCH_CHECK(carry.dim() == 4 && carry.scalar_type() == at::kFloat, "carry must be float32 (S, batch, dim, N)");
    const int64_t S = carry.size(0), Bs = carry.size(1), Dm = carry.size(2), N = carry.size(3);
    TORCH_CHECK(carry[0].is_contiguous(), "each carry slice must be contiguous");
    TORCH_CHECK(delta_sum.is_cuda() && delta_sum.scalar_type() == at::kFloat && delta_sum.dim() == 3 &&
                    delta_sum.size(0) == S && delta_sum.size(1) == Bs && delta_sum.size(2) == Dm &&
                    delta_sum[0].is_contiguous(),
                "delta_sum must be float32 (S, batch, dim)");
    TORCH_CHECK(A.is_cuda() && A.scalar_type() == at::kFloat && A.dim() == 2 && A.size(0) == Dm && A.size(1) == N &&
                    A.stride(1) == 1,
                "A must be float32 (dim, N)");
    c10::cuda::CUDAGuard guard(carry.device());
    ssm_carry_args a;
    memset(&a, 0, sizeof(a));
    a.batch = Bs; a.dim = Dm; a.dstate = N; a.nslices = S; a.reverse = reverse;
    a.A = A.data_ptr<float>(); a.A_dim_stride = A.stride(0);
    a.carry = carry.data_ptr<float>(); a.carry_slice_stride = carry.stride(0);
    a.delta_sum = delta_sum.data_ptr<float>(); a.delta_sum_slice_stride = delta_sum.stride(0);
    if (start) {
        TORCH_CHECK(start->is_cuda() && start->scalar_type() == at::kFloat && start->dim() == 4 &&
                        start->size(1) == Bs && start->size(2) == Dm && start->size(3) == N &&
                        (*start)[0].is_contiguous(),
                    "start must be float32 (R, batch, dim, N)");
        a.start = start->data_ptr<float>(); a.start_stride = start->stride(0); a.nstart = (int32_t)start->size(0);
    }
    at::Tensor result = at::empty({reverse ? S : S + 1, Bs, Dm, N}, carry.options());
    a.result = result.data_ptr<float>();
    ok(ssm_scan_carry_compose(&a, at::cuda::getCurrentCUDAStream().stream()));
    return result;
}

// One decode step; writes state_out (may be the same tensor as state) and returns out.
at::Tensor state_update(const at::Tensor& state, const at::Tensor& state_out, const at::Tensor& x,
                        const at::Tensor& dt, const at::Tensor& A, const at::Tensor& Bm, const at::Tensor& Cm,
                        const std::optional<at::Tensor>& D, const std::optional<at::Tensor>& z,
                        const std::optional<at::Tensor>& dt_bias, bool dt_softplus) {
    check_cuda(state, "h");
    TORCH_CHECK(state.dim() == 3, "h must be a 3D tensor");
    const int64_t Bs = state.size(0), Dm = state.size(1), N = state.size(2);
    TORCH_CHECK(N <= 256, "selective_update only supports state_dim <= 256");
    TORCH_CHECK(state.scalar_type() == at::kFloat, "h must be float32 tensor");
    TORCH_CHECK(state.stride(2) == 1, "h must be contiguous along the state dimension");
    TORCH_CHECK(state_out.sizes() == state.sizes() && state_out.scalar_type() == at::kFloat &&
                    state_out.stride(2) == 1 && state_out.is_cuda(),
                "state_out must match h");
    check_cuda(x, "u");
    const int32_t dtc = dtype_code(x);
    for (auto* t : {&x, &dt}) {
        TORCH_CHECK(t->is_cuda() && t->dim() == 2 && t->size(0) == Bs && t->size(1) == Dm && t->stride(1) == 1,
                    "u and delta must have shape (batch_size, num_channels)");
        TORCH_CHECK(t->scalar_type() == x.scalar_type(), "u and delta must share a dtype");
    }
    TORCH_CHECK(A.is_cuda() && A.scalar_type() == at::kFloat && A.dim() == 2 && A.size(0) == Dm && A.size(1) == N &&
                    A.stride(1) == 1,
                "A must be float32 of shape (num_channels, state_dim)");
    for (auto* t : {&Bm, &Cm}) {
        TORCH_CHECK(t->is_cuda() && t->dim() == 2 && t->size(0) == Bs && t->size(1) == N && t->stride(1) == 1,
                    "B and C must have shape (batch_size, state_dim)");
        TORCH_CHECK(t->scalar_type() == x.scalar_type(), "B and C must have the dtype of u");
    }
    if (D) { check_f32(*D, "D", {Dm}); TORCH_CHECK(D->is_contiguous(), "D must be contiguous"); }
    if (dt_bias) { check_f32(*dt_bias, "delta_bias", {Dm}); TORCH_CHECK(dt_bias->is_contiguous(), "delta_bias must be contiguous"); }
    if (z) TORCH_CHECK(z->is_cuda() && z->sizes() == x.sizes() && z->stride(1) == 1 && z->scalar_type() == x.scalar_type(),
                       "z must match x");
    c10::cuda::CUDAGuard guard(state.device());
    at::Tensor out = at::empty({Bs, Dm}, x.options());
    ssm_state_update_args a;
    memset(&a, 0, sizeof(a));
    a.batch = Bs; a.dim = Dm; a.dstate = N; a.dtype = dtc; a.dt_softplus = dt_softplus;
    a.state = state.data_ptr<float>(); a.state_batch_stride = state.stride(0); a.state_dim_stride = state.stride(1);
    a.state_out = state_out.data_ptr<float>();
    a.state_out_batch_stride = state_out.stride(0); a.state_out_dim_stride = state_out.stride(1);
    a.x = x.data_ptr(); a.x_batch_stride = x.stride(0);
    a.dt = dt.data_ptr(); a.dt_batch_stride = dt.stride(0);
    a.A = A.data_ptr<float>(); a.A_dim_stride = A.stride(0);
    a.B = Bm.data_ptr(); a.B_batch_stride = Bm.stride(0);
    a.C = Cm.data_ptr(); a.C_batch_stride = Cm.stride(0);
    a.D = ptr<const float>(D);
    if (z) { a.z = z->data_ptr(); a.z_batch_stride = z->stride(0); }
    a.dt_bias = ptr<const float>(dt_bias);
    a.out = out.data_ptr(); a.out_batch_stride = out.stride(0);
    a.launch_flags = SSM_LAUNCH_PDL;   // overlap the launch with the previous kernel's tail
    ok(ssm_state_update(&a, at::cuda::getCurrentCUDAStream().stream()));
    return out;
}

// ---- causal depthwise conv1d ------------------------------------------------------------------
void check_conv_weight(const at::Tensor& w, int64_t D) {
    check_cuda(w, "weight");
    TORCH_CHECK(w.scalar_type() == at::kFloat && w.dim() == 2 && w.size(0) == D && w.stride(1) == 1,
                "weight must be float32 of shape (dim, width) with unit width stride");
    TORCH_CHECK(w.size(1) >= 2 && w.size(1) <= 4, "conv width must be 2, 3 or 4");
}

ssm_conv1d_args conv_args(const at::Tensor& x, const at::Tensor& w, const std::optional<at::Tensor>& bias,
                          bool silu) {
    ssm_conv1d_args a;
    memset(&a, 0, sizeof(a));
    a.batch = x.size(0); a.dim = x.size(1); a.seqlen = x.dim() == 3 ? x.size(2) : 0; a.width = w.size(1);
    a.dtype = dtype_code(x); a.silu = silu;
    a.x = x.data_ptr(); a.x_batch_stride = x.stride(0); a.x_dim_stride = x.dim() == 3 ? x.stride(1) : x.stride(1);
    a.weight = w.data_ptr<float>(); a.weight_dim_stride = w.stride(0);
    if (bias) {
        check_f32(*bias, "conv bias", {x.size(1)});
        TORCH_CHECK(bias->is_contiguous(), "conv bias must be contiguous");
        a.bias = bias->data_ptr<float>();
    }
    return a;
}

// out = act(conv(x)) (+ the decode context at `length` when want_state).  Returns [out, state?].
std::vector<at::Tensor> conv1d_fwd(const at::Tensor& x, const at::Tensor& w, const std::optional<at::Tensor>& bias,
                                   bool silu, const std::optional<at::Tensor>& length, bool want_state) {
    check_cuda(x, "x");
    TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1, "x must be (batch, dim, seqlen) with unit sequence stride");
    check_conv_weight(w, x.size(1));
    c10::cuda::CUDAGuard guard(x.device());
    ssm_conv1d_args a = conv_args(x, w, bias, silu);
    at::Tensor out = at::empty(x.sizes(), x.options());
    a.out = out.data_ptr(); a.out_batch_stride = out.stride(0); a.out_dim_stride = out.stride(1);
    at::Tensor st;
    if (want_state) {
        st = at::empty({x.size(0), x.size(1), w.size(1) - 1}, x.options());
        a.state = st.data_ptr(); a.state_batch_stride = st.stride(0); a.state_dim_stride = st.stride(1);
        if (length) {
            TORCH_CHECK(length->is_cuda() && length->scalar_type() == at::kLong && length->dim() == 1 &&
                            length->size(0) == x.size(0) && length->is_contiguous(),
                        "length must be a contiguous CUDA long tensor of shape (batch,)");
            a.length = length->data_ptr<int64_t>();
        }
    }
    ok(ssm_conv1d_fwd(&a, at::cuda::getCurrentCUDAStream().stream()));
    return {out, st};
}

// Returns [dx, dweight, dbias?].
std::vector<at::Tensor> conv1d_bwd(const at::Tensor& x, const at::Tensor& w, const std::optional<at::Tensor>& bias,
                                   bool silu, const at::Tensor& dout) {
    check_cuda(x, "x");
    TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1, "x must be (batch, dim, seqlen) with unit sequence stride");
    check_conv_weight(w, x.size(1));
    check_bdl(dout, "dout", x.size(0), x.size(1), x.size(2), x.scalar_type());
    c10::cuda::CUDAGuard guard(x.device());
    ssm_conv1d_args a = conv_args(x, w, bias, silu);
    at::Tensor dx = at::empty(x.sizes(), x.options());
    at::Tensor dw = at::empty(w.sizes(), w.options());
    at::Tensor db = bias ? at::empty({x.size(1)}, w.options()) : at::Tensor();
    a.dout = dout.data_ptr(); a.dout_batch_stride = dout.stride(0); a.dout_dim_stride = dout.stride(1);
    a.dx = dx.data_ptr(); a.dx_batch_stride = dx.stride(0); a.dx_dim_stride = dx.stride(1);
    a.dweight = dw.data_ptr<float>(); a.dweight_dim_stride = dw.stride(0);
    a.dbias = bias ? db.data_ptr<float>() : nullptr;
    const size_t n = ssm_conv1d_bwd_workspace_size(&a);
    TORCH_CHECK(n > 0, ssm_last_error());
    at::Tensor ws = at::empty({(int64_t)n}, x.options().dtype(at::kByte));
    ok(ssm_conv1d_bwd(&a, ws.data_ptr(), n, at::cuda::getCurrentCUDAStream().stream()));
    return {dx, dw, db};
}

// One decode step; `state` (batch, dim, width-1) is updated in place.  Returns out (batch, dim).
at::Tensor conv1d_update(const at::Tensor& x, const at::Tensor& state, const at::Tensor& w,
                         const std::optional<at::Tensor>& bias, bool silu) {
    check_cuda(x, "x");
    TORCH_CHECK(x.dim() == 2, "x must be (batch, dim)");
    check_conv_weight(w, x.size(1));
    check_cuda(state, "conv_state");
    TORCH_CHECK(state.dim() == 3 && state.size(0) == x.size(0) && state.size(1) == x.size(1) &&
                    state.size(2) == w.size(1) - 1 && state.stride(2) == 1 && state.scalar_type() == x.scalar_type(),
                "conv_state must be (batch, dim, width - 1) of x's dtype with unit innermost stride");
    c10::cuda::CUDAGuard guard(x.device());
    ssm_conv1d_args a = conv_args(x, w, bias, silu);
    a.x_dim_stride = x.stride(1);
    at::Tensor out = at::empty(x.sizes(), x.options());
    a.out = out.data_ptr(); a.out_batch_stride = out.stride(0); a.out_dim_stride = out.stride(1);
    a.state = state.data_ptr(); a.state_batch_stride = state.stride(0); a.state_dim_stride = state.stride(1);
    ok(ssm_conv1d_update(&a, at::cuda::getCurrentCUDAStream().stream()));
    return out;
}

int64_t check_device_error() {
    int code = 0;
    ssm_check_device_error(&code, at::cuda::getCurrentCUDAStream().stream());
    return code;
}

}  // namespace

PYBIND11_MODULE(_C, m) {
    m.doc() = "torch binding of the ssm_b200 C ABI";
    m.def("scan_fwd", &scan_fwd, "selective scan forward");
    m.def("scan_bwd", &scan_bwd, "selective scan backward");
    m.def("scan_fwd_out", &scan_fwd_out, "selective scan forward into given outputs");
    m.def("scan_bwd_out", &scan_bwd_out, "selective scan backward into given outputs");
    m.def("chunk_state_fwd", &chunk_state_fwd, "per-row end state from a zero start, and sum of delta");
    m.def("chunk_state_bwd", &chunk_state_bwd, "per-row gradient into the preceding state");
    m.def("carry_compose", &carry_compose, "fold per-slice carries");
    m.def("conv1d_fwd", &conv1d_fwd, "causal depthwise conv1d (+ SiLU) forward");
    m.def("conv1d_bwd", &conv1d_bwd, "causal depthwise conv1d (+ SiLU) backward");
    m.def("conv1d_update", &conv1d_update, "causal depthwise conv1d (+ SiLU) decode step");
    m.def("ckpt_from_reference", &ckpt_from_reference, "compact checkpoints from reference chunk states");
    m.def("state_update", &state_update, "one decode step");
    m.def("ckpt_len", [](int64_t n) { return ssm_scan_ckpt_len(n); });
    m.def("version", []() { return std::string(ssm_version()); });
    m.def("check_device_error", &check_device_error, "read and clear the device error word");
}
