// PyTorch extension with the reference's op signature, over the C ABI of libnsa_sel.so.
//
//   forward(Q, K, V, sel, l_prime, BQ, cyc) -> O (fp32)
//       same arguments, meaning and errors as the reference's pybind op
//       (nsa_v2.cu:147-170, nsa_v1.cu:125-147, nsa_v0.cu:118-146): Q [B,Hq,S,D] bf16,
//       K/V [B,Hkv,S,D] bf16, sel int32 [B,Hkv,NQB,KSEL], cyc int64 [NQB*B*Hkv*2] or empty.
//       Unsupported shapes raise RuntimeError (TORCH_CHECK), as in the reference.
//   forward_lse(Q, K, V, sel, l_prime, BQ, cu_seqlens=None, scale=0, out_f32=False)
//       -> (O bf16 (or fp32), LSE fp32 [B,Hq,T]); d_qk may differ from d_v; optional varlen.
//
// The translation unit holds no device code, so it also builds when a harness compiles it
// with the reference's flags (e.g. `-arch=sm_90a`).  libnsa_sel.so is opened at first use
// from the directory of this extension, or from the package directory next to this source.
#include <dlfcn.h>
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/nsa_sel.h"

namespace {

// Error text is formatted into a per-thread buffer and raised through the `const char*` form
// of TORCH_CHECK: no std::string crosses into libtorch, so the message survives translation
// units that a harness compiles with its own flags (e.g. nvcc host code in a JIT build).
thread_local char g_msg[768];

const char* format_msg(const char* f, ...) {
  va_list ap;
  va_start(ap, f);
  vsnprintf(g_msg, sizeof(g_msg), f, ap);
  va_end(ap);
  return g_msg;
}

struct Api {
  decltype(&nsa_sel_forward) forward = nullptr;
  decltype(&nsa_sel_run) run = nullptr;
  decltype(&nsa_sel_last_error) last_error = nullptr;
  decltype(&nsa_sel_version) version = nullptr;
  decltype(&nsa_sel_select) select = nullptr;
  decltype(&nsa_sel_select_workspace_bytes) select_ws = nullptr;
};

std::string dir_of(const std::string& path) {
  const size_t p = path.find_last_of('/');
  return p == std::string::npos ? std::string(".") : path.substr(0, p);
}

const Api& api() {
  static Api a;
  static std::once_flag once;
  static std::string error;
  std::call_once(once, [] {
    std::string candidates[3];
    Dl_info info;
    if (dladdr(reinterpret_cast<void*>(&dir_of), &info) != 0 && info.dli_fname != nullptr)
      candidates[0] = dir_of(info.dli_fname) + "/libnsa_sel.so";
    candidates[1] = dir_of(dir_of(__FILE__)) + "/libnsa_sel.so";  // <pkg>/csrc/.. = <pkg>
    if (const char* env = getenv("NSA_SEL_LIBRARY")) candidates[2] = env;
    void* h = nullptr;
    for (const std::string& c : candidates) {
      if (c.empty()) continue;
      h = dlopen(c.c_str(), RTLD_NOW | RTLD_LOCAL);
      if (h != nullptr) break;
      error += c + ": " + dlerror() + "; ";
    }
    if (h == nullptr) return;
    a.forward = reinterpret_cast<decltype(a.forward)>(dlsym(h, "nsa_sel_forward"));
    a.run = reinterpret_cast<decltype(a.run)>(dlsym(h, "nsa_sel_run"));
    a.last_error = reinterpret_cast<decltype(a.last_error)>(dlsym(h, "nsa_sel_last_error"));
    a.version = reinterpret_cast<decltype(a.version)>(dlsym(h, "nsa_sel_version"));
    a.select = reinterpret_cast<decltype(a.select)>(dlsym(h, "nsa_sel_select"));
    a.select_ws = reinterpret_cast<decltype(a.select_ws)>(dlsym(h, "nsa_sel_select_workspace_bytes"));
  });
  if (!(a.forward && a.run && a.last_error && a.version && a.select && a.select_ws))
    TORCH_CHECK(false, format_msg("libnsa_sel.so could not be loaded (build it first): %s", error.c_str()));
  return a;
}

void check_inputs(const torch::Tensor& Q, const torch::Tensor& K, const torch::Tensor& V, const torch::Tensor& sel) {
  TORCH_CHECK(Q.is_cuda() && K.is_cuda() && V.is_cuda() && sel.is_cuda(), "Q, K, V and sel must be CUDA tensors");
  TORCH_CHECK(Q.scalar_type() == at::kBFloat16 && K.scalar_type() == at::kBFloat16 &&
                  V.scalar_type() == at::kBFloat16,
              "Q, K and V must be bfloat16");
  TORCH_CHECK(sel.scalar_type() == at::kInt, "sel must be int32");
  TORCH_CHECK(Q.dim() == 4 && K.dim() == 4 && V.dim() == 4 && sel.dim() == 4,
              "expected Q/K/V [B,H,S,D] and sel [B,Hkv,NQB,KSEL]");
  TORCH_CHECK(Q.is_contiguous() && K.is_contiguous() && V.is_contiguous() && sel.is_contiguous(),
              "Q, K, V and sel must be contiguous");
  TORCH_CHECK(K.size(0) == Q.size(0) && V.size(0) == Q.size(0) && sel.size(0) == Q.size(0), "batch mismatch");
  TORCH_CHECK(K.size(2) == Q.size(2) && V.size(2) == Q.size(2), "sequence length mismatch");
  TORCH_CHECK(V.size(1) == K.size(1) && sel.size(1) == K.size(1), "KV head count mismatch");
  TORCH_CHECK(K.size(3) == Q.size(3), "Q and K head dims differ");
  TORCH_CHECK(K.get_device() == Q.get_device() && V.get_device() == Q.get_device() &&
                  sel.get_device() == Q.get_device(),
              "all tensors must be on one device");
}

int32_t i32(int64_t x, const char* what) {
  if (!(x >= 0 && x < (int64_t(1) << 31))) TORCH_CHECK(false, format_msg("%s out of int32 range", what));
  return static_cast<int32_t>(x);
}

torch::Tensor forward(torch::Tensor Q, torch::Tensor K, torch::Tensor V, torch::Tensor sel, int64_t l_prime,
                      int64_t BQ, torch::Tensor cyc) {
  check_inputs(Q, K, V, sel);
  TORCH_CHECK(V.size(3) == Q.size(3), "forward() needs d_v == d_qk (use forward_lse for d_qk != d_v)");
  const Api& a = api();
  const c10::cuda::CUDAGuard guard(Q.device());
  auto O = torch::empty({Q.size(0), Q.size(1), Q.size(2), V.size(3)}, Q.options().dtype(torch::kFloat32));
  int64_t* cyc_ptr = nullptr;
  if (cyc.defined() && cyc.numel() > 0) {
    TORCH_CHECK(cyc.is_cuda() && cyc.scalar_type() == at::kLong && cyc.is_contiguous(), "cyc must be CUDA int64");
    TORCH_CHECK(cyc.numel() >= sel.size(2) * sel.size(0) * sel.size(1) * 2, "cyc must hold NQB*B*Hkv*2 entries");
    cyc_ptr = cyc.data_ptr<int64_t>();
  }
  const int rc = a.forward(Q.data_ptr(), K.data_ptr(), V.data_ptr(), sel.data_ptr<int32_t>(), O.data_ptr<float>(),
                           cyc_ptr, i32(Q.size(0), "B"), i32(Q.size(1), "Hq"), i32(K.size(1), "Hkv"),
                           i32(Q.size(2), "S"), i32(Q.size(3), "D"), i32(sel.size(2), "NQB"),
                           i32(sel.size(3), "KSEL"), i32(l_prime, "l_prime"), i32(BQ, "BQ"),
                           reinterpret_cast<nsa_stream_t>(c10::cuda::getCurrentCUDAStream().stream()));
  if (rc != NSA_OK) TORCH_CHECK(false, format_msg("nsa_sel_forward failed (%d): %s", rc, a.last_error()));
  return O;
}

std::vector<torch::Tensor> forward_lse(torch::Tensor Q, torch::Tensor K, torch::Tensor V, torch::Tensor sel,
                                       int64_t l_prime, int64_t BQ, c10::optional<torch::Tensor> cu_seqlens,
                                       double scale, bool out_f32) {
  check_inputs(Q, K, V, sel);
  const Api& a = api();
  const c10::cuda::CUDAGuard guard(Q.device());
  auto O = torch::empty({Q.size(0), Q.size(1), Q.size(2), V.size(3)},
                        Q.options().dtype(out_f32 ? torch::kFloat32 : torch::kBFloat16));
  auto L = torch::empty({Q.size(0), Q.size(1), Q.size(2)}, Q.options().dtype(torch::kFloat32));
  nsa_sel_desc d;
  memset(&d, 0, sizeof(d));
  d.q = Q.data_ptr();
  d.k = K.data_ptr();
  d.v = V.data_ptr();
  d.sel = sel.data_ptr<int32_t>();
  if (cu_seqlens.has_value() && cu_seqlens->defined()) {
    const auto& cu = *cu_seqlens;
    TORCH_CHECK(cu.is_cuda() && cu.scalar_type() == at::kInt && cu.dim() == 1 && cu.is_contiguous(),
                "cu_seqlens must be a contiguous CUDA int32 vector");
    d.cu_seqlens = cu.data_ptr<int32_t>();
    d.n_seqs = i32(cu.numel() - 1, "n_seqs");
  }
  d.o = O.data_ptr();
  d.lse = L.data_ptr<float>();
  d.batch = i32(Q.size(0), "B");
  d.heads_q = i32(Q.size(1), "Hq");
  d.heads_kv = i32(K.size(1), "Hkv");
  d.seq_len = i32(Q.size(2), "T");
  d.d_qk = i32(Q.size(3), "d_qk");
  d.d_v = i32(V.size(3), "d_v");
  d.n_qblocks = i32(sel.size(2), "NQB");
  d.n_sel = i32(sel.size(3), "KSEL");
  d.block_size = i32(l_prime, "l_prime");
  d.q_block = i32(BQ, "BQ");
  d.o_dtype = out_f32 ? NSA_DTYPE_F32 : NSA_DTYPE_BF16;
  d.scale = static_cast<float>(scale);
  const int rc = a.run(&d, reinterpret_cast<nsa_stream_t>(c10::cuda::getCurrentCUDAStream().stream()));
  if (rc != NSA_OK) TORCH_CHECK(false, format_msg("nsa_sel_run failed (%d): %s", rc, a.last_error()));
  return {O, L};
}

// Forward with the extended key visibility of nsa_sel_desc (window, compressed key map; K/V may
// have kv_len != T rows with the compressed map): returns [O (fp32), LSE].
std::vector<torch::Tensor> forward_ext(torch::Tensor Q, torch::Tensor K, torch::Tensor V, torch::Tensor sel,
                                       int64_t l_prime, int64_t BQ, int64_t window, int64_t key_map, double scale,
                                       c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> weight,
                                       bool accumulate, bool with_lse) {
  TORCH_CHECK(Q.is_cuda() && K.is_cuda() && V.is_cuda() && sel.is_cuda(), "Q, K, V and sel must be CUDA tensors");
  TORCH_CHECK(Q.scalar_type() == at::kBFloat16 && K.scalar_type() == at::kBFloat16 &&
                  V.scalar_type() == at::kBFloat16,
              "Q, K and V must be bfloat16");
  TORCH_CHECK(sel.scalar_type() == at::kInt, "sel must be int32");
  TORCH_CHECK(Q.dim() == 4 && K.dim() == 4 && V.dim() == 4 && sel.dim() == 4,
              "expected Q [B,Hq,T,d], K/V [B,Hkv,kv_len,d] and sel [B,Hkv,NQB,KSEL]");
  TORCH_CHECK(Q.is_contiguous() && K.is_contiguous() && V.is_contiguous() && sel.is_contiguous(),
              "Q, K, V and sel must be contiguous");
  TORCH_CHECK(K.size(0) == Q.size(0) && V.size(0) == Q.size(0) && sel.size(0) == Q.size(0), "batch mismatch");
  TORCH_CHECK(V.size(2) == K.size(2) && V.size(1) == K.size(1) && sel.size(1) == K.size(1), "K/V shape mismatch");
  TORCH_CHECK(K.size(3) == Q.size(3), "Q and K head dims differ");
  const Api& a = api();
  const c10::cuda::CUDAGuard guard(Q.device());
  torch::Tensor O;
  if (out.has_value()) {
    O = *out;
    TORCH_CHECK(O.is_cuda() && O.scalar_type() == at::kFloat && O.is_contiguous() && O.get_device() == Q.get_device(),
                "out must be a contiguous fp32 CUDA tensor on Q's device");
    TORCH_CHECK(O.dim() == 4 && O.size(0) == Q.size(0) && O.size(1) == Q.size(1) && O.size(2) == Q.size(2) &&
                    O.size(3) == V.size(3),
                "out must be [B, Hq, T, d_v]");
  } else {
    TORCH_CHECK(!accumulate, "accumulate needs an out tensor");
    O = torch::empty({Q.size(0), Q.size(1), Q.size(2), V.size(3)}, Q.options().dtype(torch::kFloat32));
  }
  if (weight.has_value())
    TORCH_CHECK(weight->is_cuda() && weight->scalar_type() == at::kFloat && weight->numel() >= 1 &&
                    weight->get_device() == Q.get_device(),
                "weight must be an fp32 CUDA tensor (its first element is used) on Q's device");
  torch::Tensor L = with_lse ? torch::empty({Q.size(0), Q.size(1), Q.size(2)}, Q.options().dtype(torch::kFloat32))
                             : torch::empty({0}, Q.options().dtype(torch::kFloat32));
  nsa_sel_desc d;
  memset(&d, 0, sizeof(d));
  d.q = Q.data_ptr();
  d.k = K.data_ptr();
  d.v = V.data_ptr();
  d.sel = sel.data_ptr<int32_t>();
  d.o = O.data_ptr();
  d.lse = with_lse ? L.data_ptr<float>() : nullptr;
  d.o_accumulate = accumulate ? 1 : 0;
  d.o_weight = weight.has_value() ? weight->data_ptr<float>() : nullptr;
  d.batch = i32(Q.size(0), "B");
  d.heads_q = i32(Q.size(1), "Hq");
  d.heads_kv = i32(K.size(1), "Hkv");
  d.seq_len = i32(Q.size(2), "T");
  d.kv_len = i32(K.size(2), "kv_len");
  d.d_qk = i32(Q.size(3), "d_qk");
  d.d_v = i32(V.size(3), "d_v");
  d.n_qblocks = i32(sel.size(2), "NQB");
  d.n_sel = i32(sel.size(3), "KSEL");
  d.block_size = i32(l_prime, "l_prime");
  d.q_block = i32(BQ, "BQ");
  d.window = i32(window, "window");
  d.key_map = i32(key_map, "key_map");
  d.o_dtype = NSA_DTYPE_F32;
  d.scale = static_cast<float>(scale);
  const int rc = a.run(&d, reinterpret_cast<nsa_stream_t>(c10::cuda::getCurrentCUDAStream().stream()));
  if (rc != NSA_OK) TORCH_CHECK(false, format_msg("nsa_sel_run failed (%d): %s", rc, a.last_error()));
  return {O, L};
}

// Block selection (nsa_sel_select): sel int32 [B, Hkv, T, min(n_sel, ceil(T/l_prime))].
torch::Tensor select_blocks(torch::Tensor Q, torch::Tensor K, int64_t n_sel, int64_t l_prime, int64_t cmp_block,
                            int64_t cmp_stride) {
  TORCH_CHECK(Q.is_cuda() && K.is_cuda(), "Q and K must be CUDA tensors");
  TORCH_CHECK(Q.scalar_type() == at::kBFloat16 && K.scalar_type() == at::kBFloat16, "Q and K must be bfloat16");
  TORCH_CHECK(Q.dim() == 4 && K.dim() == 4, "expected Q [B,Hq,T,d] and K [B,Hkv,T,d]");
  TORCH_CHECK(Q.is_contiguous() && K.is_contiguous(), "Q and K must be contiguous");
  TORCH_CHECK(K.size(0) == Q.size(0) && K.size(2) == Q.size(2) && K.size(3) == Q.size(3), "Q/K shape mismatch");
  const Api& a = api();
  const c10::cuda::CUDAGuard guard(Q.device());
  const int32_t B = i32(Q.size(0), "B"), Hq = i32(Q.size(1), "Hq"), Hkv = i32(K.size(1), "Hkv");
  const int32_t T = i32(Q.size(2), "T"), d = i32(Q.size(3), "d"), lp = i32(l_prime, "l_prime");
  const int64_t ws = a.select_ws(B, Hkv, T, d, lp);
  if (ws < 0) TORCH_CHECK(false, "invalid selection shape");
  const int64_t n_blk = (T + lp - 1) / lp;
  const int64_t k = std::min<int64_t>(n_sel, n_blk);
  auto work = torch::empty({std::max<int64_t>(ws / 4, 1)}, Q.options().dtype(torch::kFloat32));
  auto sel = torch::empty({Q.size(0), K.size(1), Q.size(2), std::max<int64_t>(k, 1)}, Q.options().dtype(torch::kInt));
  const int rc = a.select(Q.data_ptr(), K.data_ptr(), work.data_ptr<float>(), sel.data_ptr<int32_t>(), B, Hq, Hkv, T, d,
                          lp, i32(n_sel, "n_sel"), i32(cmp_block, "cmp_block"), i32(cmp_stride, "cmp_stride"),
                          reinterpret_cast<nsa_stream_t>(c10::cuda::getCurrentCUDAStream().stream()));
  if (rc != NSA_OK) TORCH_CHECK(false, format_msg("nsa_sel_select failed (%d): %s", rc, a.last_error()));
  return sel;
}

int64_t library_version() { return api().version(); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 NSA selected-branch forward (sm_100a) with the nsa-hopper op signature";
  m.def("forward", &forward, "forward(Q, K, V, sel, l_prime, BQ, cyc) -> O (fp32)");
  m.def("forward_lse", &forward_lse, "forward_lse(Q, K, V, sel, l_prime, BQ, cu_seqlens, scale, out_f32) -> [O, LSE]",
        py::arg("Q"), py::arg("K"), py::arg("V"), py::arg("sel"), py::arg("l_prime"), py::arg("BQ"),
        py::arg("cu_seqlens") = py::none(), py::arg("scale") = 0.0, py::arg("out_f32") = false);
  m.def("forward_ext", &forward_ext,
        "forward_ext(Q, K, V, sel, l_prime, BQ, window, key_map, scale, out, weight, accumulate, with_lse) -> "
        "[O fp32, LSE]",
        py::arg("Q"), py::arg("K"), py::arg("V"), py::arg("sel"), py::arg("l_prime"), py::arg("BQ"),
        py::arg("window") = 0, py::arg("key_map") = 0, py::arg("scale") = 0.0, py::arg("out") = py::none(),
        py::arg("weight") = py::none(), py::arg("accumulate") = false, py::arg("with_lse") = true);
  m.def("select_blocks", &select_blocks, "select_blocks(Q, K, n_sel, l_prime, cmp_block, cmp_stride) -> sel int32",
        py::arg("Q"), py::arg("K"), py::arg("n_sel"), py::arg("l_prime"), py::arg("cmp_block") = 32,
        py::arg("cmp_stride") = 16);
  m.def("library_version", &library_version);
}
