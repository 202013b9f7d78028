// Python bindings of the sm_100a kernels (module osp_next_b200.ops._C).
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <map>
#include <mutex>
#include <utility>

#include "tma_host.h"

namespace osp {
void gemm(const at::Tensor& a, const at::Tensor& b, const c10::optional<at::Tensor>& bias, at::Tensor& out,
          int64_t act, const c10::optional<at::Tensor>& resid, const c10::optional<at::Tensor>& gate,
          const c10::optional<at::Tensor>& dest_row, int64_t rows_per_batch, int64_t n_out);
void gemm_dual(const at::Tensor& a, const at::Tensor& b, const at::Tensor& a2, const at::Tensor& b2,
               const c10::optional<at::Tensor>& bias, at::Tensor& out, int64_t act,
               const c10::optional<at::Tensor>& resid, const c10::optional<at::Tensor>& gate,
               const c10::optional<at::Tensor>& dest_row, int64_t rows_per_batch, int64_t n_out);
void gemm_t(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, bool a_mn, bool b_mn);
void gemm_gelu_aux(const at::Tensor& a, const at::Tensor& b, const c10::optional<at::Tensor>& bias, at::Tensor& out,
                   at::Tensor& aux, const c10::optional<at::Tensor>& a2, const c10::optional<at::Tensor>& b2);
void ln_modulate_bwd(const at::Tensor& x, const at::Tensor& dy, const at::Tensor& scale, at::Tensor& dx,
                     at::Tensor& dscale_part, at::Tensor& dshift_part, double eps);
void gated_add_fwd(const at::Tensor& resid, const at::Tensor& y, const c10::optional<at::Tensor>& gate,
                   at::Tensor& out);
void gated_add_bwd(const at::Tensor& dout, const at::Tensor& y, const at::Tensor& gate, at::Tensor& dy,
                   at::Tensor& dgate_part);
void qk_norm_rope_bwd(const at::Tensor& raw, const at::Tensor& g, const at::Tensor& w, const at::Tensor& pos,
                      const at::Tensor& freqs, at::Tensor& dqkv, at::Tensor& dw_part, int64_t part, int64_t B,
                      int64_t n, int64_t C, int64_t D, double eps);
void gelu_tanh_bwd(const at::Tensor& dh, const at::Tensor& pre, at::Tensor& dpre);
void bias_grad(const at::Tensor& g, at::Tensor& part);
void rms_norm_bwd(const at::Tensor& x, const at::Tensor& dy, const c10::optional<at::Tensor>& w, at::Tensor& dx,
                  at::Tensor& dw_part, double eps);
void ln_modulate(const at::Tensor& x, const c10::optional<at::Tensor>& shift, const c10::optional<at::Tensor>& scale,
                 const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& b, at::Tensor& out, double eps);
void rms_norm(const at::Tensor& x, const c10::optional<at::Tensor>& w, at::Tensor& out, double eps);
void qk_norm_rope(at::Tensor& qkv, const at::Tensor& wq, const at::Tensor& wk, const at::Tensor& pos,
                  const at::Tensor& freqs, int64_t num_heads, double eps);
void attention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& seg_q,
                   const at::Tensor& seg_k, at::Tensor& out, at::Tensor& lse, double scale, int64_t max_q);
void attention_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                   const at::Tensor& dout, const at::Tensor& lse, const at::Tensor& seg_q, const at::Tensor& seg_k,
                   at::Tensor& dq, at::Tensor& dk, at::Tensor& dv, at::Tensor& delta, double scale, int64_t max_q,
                   int64_t max_k);
void cfg_euler(const at::Tensor& lat, const at::Tensor& cond, const at::Tensor& unc, at::Tensor& out, double g,
               double dt);
void hif8_round(const at::Tensor& x, at::Tensor& out, double s);
void hif8_qdq(const at::Tensor& x, at::Tensor& out, double scale_max);
void adamw(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v, double lr, double b1, double b2,
           double eps, double wd, int64_t step, double gscale);
void sde_step(const at::Tensor& x, const at::Tensor& v, const c10::optional<at::Tensor>& xi,
              const c10::optional<at::Tensor>& prev_in, at::Tensor& prev_out, const c10::optional<at::Tensor>& mean_out,
              at::Tensor& logp, double sigma, double dt, double smin, double smax);
void wait_probe(int64_t mode, const at::Tensor& flag, double limit_s);
void gemm_p2p(const at::Tensor& a, const at::Tensor& b, const c10::optional<at::Tensor>& bias,
              const at::Tensor& resid, const c10::optional<at::Tensor>& gate, const at::Tensor& dest_rank,
              const at::Tensor& dest_row, const at::Tensor& out_ptrs, int64_t rows_per_batch, int64_t n_stride);
std::tuple<int64_t, std::string> p2p_alloc(int64_t bytes);
int64_t p2p_open(const std::string& handle);
void p2p_close(int64_t ptr);
void p2p_free(int64_t ptr);
at::Tensor p2p_view(int64_t ptr, std::vector<int64_t> shape, at::ScalarType dtype, int64_t device);
void p2p_barrier(const at::Tensor& flag_ptrs, int64_t rank, int64_t world, int64_t epoch, double limit_s);
void p2p_pull(at::Tensor& out, const at::Tensor& ptrs, const at::Tensor& rank, const at::Tensor& off, int64_t R,
              int64_t chunk_bytes, bool sum);
void p2p_barrier_tagged(const at::Tensor& flag_ptrs, int64_t rank, int64_t world, int64_t epoch, int64_t tag,
                        double limit_s);
void p2p_gather(const at::Tensor& bases, int64_t off, int64_t shard_bytes, int64_t rank, int64_t world,
                int64_t abort_ptr);
void p2p_reduce_scatter_f32(at::Tensor& out, const at::Tensor& bases, int64_t off, int64_t shard_elems, int64_t rank,
                            int64_t world, double scale, int64_t abort_ptr);
void p2p_reduce_scatter_bf16(at::Tensor& out, const at::Tensor& bases, int64_t off, int64_t shard_elems, int64_t rank,
                            int64_t world, double scale, int64_t abort_ptr);

static int* g_err[kMaxDevices] = {nullptr};
static std::mutex g_err_mu;

static void check_device(int device) {
  TORCH_CHECK(device >= 0 && device < kMaxDevices, "device ordinal ", device, " out of range [0, ", kMaxDevices, ")");
}

int* error_word(int device) {
  check_device(device);
  std::lock_guard<std::mutex> lk(g_err_mu);
  if (!g_err[device]) {
    c10::cuda::CUDAGuard guard(device);
    C10_CUDA_CHECK(cudaMalloc(&g_err[device], sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(g_err[device], 0, sizeof(int)));
  }
  return g_err[device];
}

int num_sms(int device) {
  check_device(device);
  static int cache[kMaxDevices] = {0};
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (!cache[device]) C10_CUDA_CHECK(cudaDeviceGetAttribute(&cache[device], cudaDevAttrMultiProcessorCount, device));
  return cache[device];
}

void smem_opt_in(const void* kernel, int bytes) {
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  check_device(dev);
  static std::map<std::pair<const void*, int>, int> done;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  int& have = done[std::make_pair(kernel, dev)];
  if (have >= bytes) return;
  C10_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  have = bytes;
}

// Read (and optionally clear) the first error code recorded by a bounded device wait.
int64_t get_error(int64_t device, bool clear) {
  int* w = error_word((int)device);
  int h = 0;
  c10::cuda::CUDAGuard guard((int)device);
  C10_CUDA_CHECK(cudaDeviceSynchronize());
  C10_CUDA_CHECK(cudaMemcpy(&h, w, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear) C10_CUDA_CHECK(cudaMemset(w, 0, sizeof(int)));
  return h;
}
}  // namespace osp

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "OSP-Next B200 kernels (sm_100a: tcgen05 GEMM + flash attention, fused elementwise)";
  m.def("gemm", &osp::gemm);
  m.def("gemm_dual", &osp::gemm_dual);
  m.def("ln_modulate", &osp::ln_modulate);
  m.def("rms_norm", &osp::rms_norm);
  m.def("qk_norm_rope", &osp::qk_norm_rope);
  m.def("gemm_t", &osp::gemm_t);
  m.def("gemm_gelu_aux", &osp::gemm_gelu_aux, pybind11::arg("a"), pybind11::arg("b"), pybind11::arg("bias"),
        pybind11::arg("out"), pybind11::arg("aux"), pybind11::arg("a2") = pybind11::none(),
        pybind11::arg("b2") = pybind11::none());
  m.def("ln_modulate_bwd", &osp::ln_modulate_bwd);
  m.def("gated_add_fwd", &osp::gated_add_fwd);
  m.def("gated_add_bwd", &osp::gated_add_bwd);
  m.def("qk_norm_rope_bwd", &osp::qk_norm_rope_bwd);
  m.def("gelu_tanh_bwd", &osp::gelu_tanh_bwd);
  m.def("bias_grad", &osp::bias_grad);
  m.def("rms_norm_bwd", &osp::rms_norm_bwd);
  m.def("attention_fwd", &osp::attention_fwd);
  m.def("attention_bwd", &osp::attention_bwd);
  m.def("cfg_euler", &osp::cfg_euler);
  m.def("hif8_round", &osp::hif8_round);
  m.def("hif8_qdq", &osp::hif8_qdq);
  m.def("adamw", &osp::adamw);
  m.def("sde_step", &osp::sde_step);
  m.def("wait_probe", &osp::wait_probe);
  m.def("gemm_p2p", &osp::gemm_p2p);
  m.def("p2p_alloc", [](int64_t bytes) {
    auto r = osp::p2p_alloc(bytes);
    return pybind11::make_tuple(std::get<0>(r), pybind11::bytes(std::get<1>(r)));
  });
  m.def("p2p_open", [](pybind11::bytes h) { return osp::p2p_open(std::string(h)); });
  m.def("p2p_close", &osp::p2p_close);
  m.def("p2p_free", &osp::p2p_free);
  m.def("p2p_view", &osp::p2p_view);
  m.def("p2p_barrier", &osp::p2p_barrier);
  m.def("p2p_pull", &osp::p2p_pull);
  m.def("p2p_barrier_tagged", &osp::p2p_barrier_tagged);
  m.def("p2p_gather", &osp::p2p_gather);
  m.def("p2p_reduce_scatter_f32", &osp::p2p_reduce_scatter_f32);
  m.def("p2p_reduce_scatter_bf16", &osp::p2p_reduce_scatter_bf16);
  m.def("get_error", &osp::get_error, pybind11::arg("device"), pybind11::arg("clear") = true);
}
