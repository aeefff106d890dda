// fusionpass_b200._fpkern: the torch C++ extension over the C ABI of libfpkern.so.
//
// The plan runtime's fused steps reach the kernels here (the reference launches
// them from python/fusionpass/kernels.py:288-333 as Triton kernels):
//
//   attention(q, k, v, out, desc)   O = softmax(scale * Q K^T) V into `out`
//   chain(inputs, out, desc)        one fused elementwise chain into `out`
//
// Both validate devices, dtypes, shapes and strides, enqueue on torch's current
// CUDA stream of the tensors' device (c10::cuda::getCurrentCUDAStream), and
// raise instead of falling back: ValueError for arguments that cannot describe
// a launch, RuntimeError carrying fpk_status_string() for a status the library
// returns.  No tensor is allocated or copied here; the caller owns `out`.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cstring>
#include <string>

#include "fpkern.h"

namespace {

[[noreturn]] void value_error(const std::string& msg) { throw pybind11::value_error(msg); }

void check_status(int rc, const char* what) {
  if (rc != FPK_OK)
    throw std::runtime_error(std::string(what) + ": " + fpk_status_string(rc) + " (status " + std::to_string(rc) +
                             ")");
}

int32_t dtype_code(const at::Tensor& t) {
  if (t.scalar_type() == at::kHalf) return FPK_F16;
  if (t.scalar_type() == at::kFloat) return FPK_F32;
  value_error(std::string("unsupported dtype ") + c10::toString(t.scalar_type()) + " (f16 and f32 only)");
}

void require_cuda(const at::Tensor& t, const char* what) {
  if (!t.defined() || !t.is_cuda())
    throw std::runtime_error(std::string(what) +
                             ": fused steps run only in libfpkern.so on a CUDA device; there is no CPU path");
}

void* stream_of(const at::Tensor& t) { return c10::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

// (batch, heads, seq, head_dim) and element strides (b, h, s) of a [..., S, D]
// tensor with unit last stride whose leading dims flatten to one stride.
struct Bhsd {
  int64_t b, h, s, d;
  int64_t st[3];
};

Bhsd bhsd(const at::Tensor& t, const char* name) {
  if (t.dim() < 3) value_error(std::string(name) + ": attention tensors need rank >= 3 ([batch..., S, D])");
  if (t.stride(-1) != 1) value_error(std::string(name) + ": the last dim must have unit stride");
  Bhsd r;
  r.s = t.size(-2);
  r.d = t.size(-1);
  if (t.dim() == 3) {
    r.b = 1;
    r.h = t.size(0);
    r.st[0] = t.size(0) * t.stride(0);
    r.st[1] = t.stride(0);
    r.st[2] = t.stride(1);
    return r;
  }
  r.h = t.size(-3);
  r.b = 1;
  for (int64_t i = 0; i < t.dim() - 3; ++i) r.b *= t.size(i);
  for (int64_t i = t.dim() - 5; i >= 0; --i)
    if (t.size(i) > 1 && t.stride(i) != t.stride(i + 1) * t.size(i + 1))
      value_error(std::string(name) + ": the dims before heads must flatten to one stride");
  r.st[0] = t.stride(-4);
  r.st[1] = t.stride(-3);
  r.st[2] = t.stride(-2);
  return r;
}

at::Tensor attention(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor out,
                     const pybind11::dict& desc, int64_t flags) {
  require_cuda(q, "attention");
  require_cuda(k, "attention");
  require_cuda(v, "attention");
  require_cuda(out, "attention");
  if (!(q.sizes() == k.sizes() && q.sizes() == v.sizes() && q.sizes() == out.sizes()))
    value_error("q, k, v and out must share one shape (FusedAttentionOp contract)");
  if (!(q.scalar_type() == k.scalar_type() && q.scalar_type() == v.scalar_type() &&
        q.scalar_type() == out.scalar_type()))
    value_error("q, k, v and out must share one dtype");
  if (k.device() != q.device() || v.device() != q.device() || out.device() != q.device())
    value_error("q, k, v and out must be on one device");
  if (!desc.contains("scale")) value_error("attention descriptor has no 'scale'");
  const Bhsd bq = bhsd(q, "q"), bk = bhsd(k, "k"), bv = bhsd(v, "v"), bo = bhsd(out, "out");
  if (desc.contains("head_dim") && desc["head_dim"].cast<int64_t>() != bq.d)
    value_error("descriptor head_dim " + std::to_string(desc["head_dim"].cast<int64_t>()) + " != tensor head dim " +
                std::to_string(bq.d));
  fpk_attn_desc d;
  std::memset(&d, 0, sizeof(d));
  d.size = sizeof(d);
  d.version = FPK_ABI_VERSION;
  d.dtype = dtype_code(q);
  d.head_dim = static_cast<int32_t>(bq.d);
  d.batch = bq.b;
  d.heads = bq.h;
  d.seq_len = bq.s;
  d.scale = desc["scale"].cast<float>();
  d.flags = static_cast<uint32_t>(flags);
  for (int i = 0; i < 3; ++i) {
    d.q_strides[i] = bq.st[i];
    d.k_strides[i] = bk.st[i];
    d.v_strides[i] = bv.st[i];
    d.o_strides[i] = bo.st[i];
  }
  const c10::cuda::CUDAGuard guard(q.device());
  check_status(fpk_attention_fwd(&d, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), stream_of(q)),
               "fpk_attention_fwd");
  return out;
}

// Broadcast mode of one chain operand on a [rows, cols] output: the descriptor's
// declaration when it has one, else the operand's shape decides (as torch would
// place it); an operand that fits two modes on a square output must be declared.
int32_t bcast_code(const at::Tensor& t, int64_t rows, int64_t cols, const pybind11::handle& declared) {
  const int64_t n = t.numel();
  if (!declared.is_none()) {
    const std::string b = declared.cast<std::string>();
    int32_t code;
    int64_t want;
    if (b == "full") { code = FPK_BCAST_FULL; want = rows * cols; }
    else if (b == "col") { code = FPK_BCAST_COL; want = cols; }
    else if (b == "row") { code = FPK_BCAST_ROW; want = rows; }
    else if (b == "scalar") { code = FPK_BCAST_SCALAR; want = 1; }
    else value_error("unknown broadcast mode '" + b + "'");
    if (n != want)
      value_error("operand with " + std::to_string(n) + " elements does not match broadcast '" + b + "' of a [" +
                  std::to_string(rows) + ", " + std::to_string(cols) + "] chain");
    return code;
  }
  if (n == rows * cols) return FPK_BCAST_FULL;
  if (n == 1) return FPK_BCAST_SCALAR;
  if (n == cols && n == rows) {
    if (t.dim() >= 2 && t.size(-1) == 1) return FPK_BCAST_ROW;
    if (t.dim() == 1 || (t.size(-1) == cols && t.size(-2) == 1)) return FPK_BCAST_COL;
    value_error("operand is ambiguous on a square chain: declare its broadcast in the descriptor's 'inputs'");
  }
  if (n == cols) return FPK_BCAST_COL;
  if (n == rows) return FPK_BCAST_ROW;
  value_error("operand with " + std::to_string(n) + " elements cannot broadcast onto [" + std::to_string(rows) + ", " +
              std::to_string(cols) + "]");
}

int32_t opcode_of(const std::string& op) {
  if (op == "add") return FPK_OP_ADD;
  if (op == "mul") return FPK_OP_MUL;
  if (op == "scale") return FPK_OP_SCALE;
  if (op == "relu") return FPK_OP_RELU;
  if (op == "exp") return FPK_OP_EXP;
  if (op == "softmax") return FPK_OP_SOFTMAX;
  if (op == "gelu") return FPK_OP_GELU;
  value_error("unsupported op in chain: " + op);
}

at::Tensor chain(const std::vector<at::Tensor>& inputs, at::Tensor out, const pybind11::dict& desc, int64_t flags,
                 const pybind11::object& mode) {
  require_cuda(out, "chain");
  if (!out.is_contiguous()) value_error("out must be contiguous");
  const int n_in = static_cast<int>(inputs.size());
  if (n_in < 1 || n_in > FPK_CHAIN_MAX_INPUTS)
    value_error("chain needs 1.." + std::to_string(FPK_CHAIN_MAX_INPUTS) + " inputs, got " + std::to_string(n_in));
  const pybind11::list ops = desc["ops"].cast<pybind11::list>();
  const int n_ops = static_cast<int>(ops.size());
  if (n_ops < 1 || n_ops > FPK_CHAIN_MAX_OPS)
    value_error("chain needs 1.." + std::to_string(FPK_CHAIN_MAX_OPS) + " ops, got " + std::to_string(n_ops));
  const int64_t cols = out.dim() > 0 ? out.size(-1) : 1;
  const int64_t rows = cols > 0 ? out.numel() / cols : 0;
  pybind11::list specs;
  if (desc.contains("inputs")) specs = desc["inputs"].cast<pybind11::list>();
  if (specs.size() != 0 && static_cast<int>(specs.size()) != n_in)
    value_error("descriptor lists " + std::to_string(specs.size()) + " inputs, step has " + std::to_string(n_in));
  fpk_chain_desc d;
  std::memset(&d, 0, sizeof(d));
  d.size = sizeof(d);
  d.version = FPK_ABI_VERSION;
  const std::string m = !mode.is_none() ? mode.cast<std::string>()
                                        : (desc.contains("mode") ? desc["mode"].cast<std::string>() : "flat");
  d.mode = m == "rows" ? FPK_CHAIN_ROWS : FPK_CHAIN_FLAT;
  d.out_dtype = dtype_code(out);
  d.rows = rows;
  d.cols = cols;
  d.n_inputs = n_in;
  d.n_ops = n_ops;
  d.result = desc["result"].cast<int32_t>();
  d.flags = static_cast<uint32_t>(flags);
  const void* ptrs[FPK_CHAIN_MAX_INPUTS];
  for (int i = 0; i < n_in; ++i) {
    const at::Tensor& t = inputs[i];
    require_cuda(t, "chain");
    if (t.device() != out.device()) value_error("all chain operands must be on one device");
    if (!t.is_contiguous()) value_error("chain operand " + std::to_string(i) + " must be contiguous");
    d.in_dtype[i] = dtype_code(t);
    pybind11::object declared = pybind11::none();
    if (specs.size() != 0) {
      const pybind11::dict spec = specs[i].cast<pybind11::dict>();
      if (spec.contains("bcast")) declared = spec["bcast"];
    }
    d.in_bcast[i] = bcast_code(t, rows, cols, declared);
    ptrs[i] = t.data_ptr();
  }
  for (int k = 0; k < n_ops; ++k) {
    const pybind11::dict op = ops[k].cast<pybind11::dict>();
    d.ops[k].opcode = opcode_of(op["op"].cast<std::string>());
    d.ops[k].src_a = op["a"].cast<int32_t>();
    d.ops[k].src_b = op.contains("b") ? op["b"].cast<int32_t>() : -1;
    d.ops[k].imm = op.contains("imm") ? op["imm"].cast<float>() : 0.0f;
  }
  const c10::cuda::CUDAGuard guard(out.device());
  check_status(fpk_chain_fwd(&d, ptrs, n_in, out.data_ptr(), stream_of(out)), "fpk_chain_fwd");
  return out;
}

}  // namespace

// LayerNorm over the last axis of a contiguous x into out (same shape and dtype); w and b
// per-column (length cols) or both undefined.  Returns false, leaving out untouched,
// when the kernel does not take the shape (cols not a multiple of 8 or above
// FPK_LN_MAX_COLS, unaligned pointers): the caller then runs its own layer_norm.
bool layer_norm(const at::Tensor& x, const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& b,
                at::Tensor out, double eps) {
  require_cuda(x, "layer_norm");
  require_cuda(out, "layer_norm");
  if (!x.is_contiguous() || !out.is_contiguous()) value_error("layer_norm: x and out must be contiguous");
  if (out.sizes() != x.sizes() || out.scalar_type() != x.scalar_type() || out.device() != x.device())
    value_error("layer_norm: out must match x in shape, dtype and device");
  if (x.dim() < 1) value_error("layer_norm: x needs at least one dim");
  const bool affine = w.has_value() && w->defined();
  if (affine != (b.has_value() && b->defined())) value_error("layer_norm: give both weight and bias, or neither");
  fpk_ln_desc d;
  std::memset(&d, 0, sizeof(d));
  d.size = sizeof(d);
  d.version = FPK_ABI_VERSION;
  d.dtype = dtype_code(x);
  d.cols = x.size(-1);
  d.rows = d.cols > 0 ? x.numel() / d.cols : 0;
  d.eps = static_cast<float>(eps);
  if (affine) {
    for (const at::Tensor* t : {&*w, &*b}) {
      require_cuda(*t, "layer_norm");
      if (t->numel() != d.cols || !t->is_contiguous() || t->scalar_type() != x.scalar_type() ||
          t->device() != x.device())
        value_error("layer_norm: weight and bias must be contiguous vectors of the last dim's size and x's dtype");
    }
  }
  const c10::cuda::CUDAGuard guard(x.device());
  const int rc = fpk_layer_norm_fwd(&d, x.data_ptr(), affine ? w->data_ptr() : nullptr,
                                    affine ? b->data_ptr() : nullptr, out.data_ptr(), stream_of(x));
  if (rc == FPK_ERR_UNSUPPORTED || rc == FPK_ERR_ALIGN) return false;
  check_status(rc, "fpk_layer_norm_fwd");
  return true;
}

// LayerNorm over the last axis of the sum of 1..4 addends (each of out's shape, or a
// vector of its last dim's size, added in order) into out.  False, leaving out
// untouched, when the kernel does not take the shape.
bool add_layer_norm(const std::vector<at::Tensor>& addends, const c10::optional<at::Tensor>& w,
                    const c10::optional<at::Tensor>& b, at::Tensor out, double eps) {
  require_cuda(out, "add_layer_norm");
  if (!out.is_contiguous() || out.dim() < 1) value_error("add_layer_norm: out must be contiguous with rank >= 1");
  if (addends.empty() || addends.size() > 4) value_error("add_layer_norm: 1 to 4 addends");
  const bool affine = w.has_value() && w->defined();
  if (affine != (b.has_value() && b->defined())) value_error("add_layer_norm: give both weight and bias, or neither");
  fpk_ln_desc d;
  std::memset(&d, 0, sizeof(d));
  d.size = sizeof(d);
  d.version = FPK_ABI_VERSION;
  d.dtype = dtype_code(out);
  d.cols = out.size(-1);
  d.rows = d.cols > 0 ? out.numel() / d.cols : 0;
  d.eps = static_cast<float>(eps);
  const void* ptrs[4];
  int32_t bc[4];
  for (size_t i = 0; i < addends.size(); ++i) {
    const at::Tensor& t = addends[i];
    require_cuda(t, "add_layer_norm");
    if (!t.is_contiguous() || t.scalar_type() != out.scalar_type() || t.device() != out.device())
      value_error("add_layer_norm: addends must be contiguous, of out's dtype and device");
    if (t.sizes() == out.sizes()) bc[i] = FPK_BCAST_FULL;
    else if (t.numel() == d.cols && t.size(-1) == d.cols) bc[i] = FPK_BCAST_COL;
    else value_error("add_layer_norm: an addend has neither out's shape nor its last dim's size");
    ptrs[i] = t.data_ptr();
  }
  if (affine) {
    for (const at::Tensor* t : {&*w, &*b}) {
      require_cuda(*t, "add_layer_norm");
      if (t->numel() != d.cols || !t->is_contiguous() || t->scalar_type() != out.scalar_type() ||
          t->device() != out.device())
        value_error("add_layer_norm: weight and bias must be contiguous vectors of the last dim's size and out's dtype");
    }
  }
  const c10::cuda::CUDAGuard guard(out.device());
  const int rc = fpk_add_layer_norm_fwd(&d, ptrs, bc, static_cast<int>(addends.size()), affine ? w->data_ptr() : nullptr,
                                        affine ? b->data_ptr() : nullptr, out.data_ptr(), stream_of(out));
  if (rc == FPK_ERR_UNSUPPORTED || rc == FPK_ERR_ALIGN) return false;
  check_status(rc, "fpk_add_layer_norm_fwd");
  return true;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "fusionpass_b200._fpkern: torch binding of libfpkern.so (sm_100a fused-step kernels)";
  m.def("version", &fpk_version, "ABI version of the loaded libfpkern.so");
  m.def("attention", &attention, "softmax(scale * q @ k^T) @ v into out on the current CUDA stream",
        pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"), pybind11::arg("out"), pybind11::arg("desc"),
        pybind11::arg("flags") = 0);
  m.def("layer_norm", &layer_norm, "LayerNorm over the last axis into out; False if the kernel does not take the shape",
        pybind11::arg("x"), pybind11::arg("weight"), pybind11::arg("bias"), pybind11::arg("out"), pybind11::arg("eps"));
  m.def("add_layer_norm", &add_layer_norm,
        "LayerNorm over the last axis of the sum of the addends into out; False if the kernel does not take the shape",
        pybind11::arg("addends"), pybind11::arg("weight"), pybind11::arg("bias"), pybind11::arg("out"),
        pybind11::arg("eps"));
  m.def("chain", &chain, "one fused elementwise chain into out on the current CUDA stream", pybind11::arg("inputs"),
        pybind11::arg("out"), pybind11::arg("desc"), pybind11::arg("flags") = 0,
        pybind11::arg("mode") = pybind11::none());
}
