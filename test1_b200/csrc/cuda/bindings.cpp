// Python bindings of the sm_100a kernel library (test1_b200._cuda).
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <string>
#include <tuple>
#include <unordered_map>
#include <utility>
#include <vector>

namespace t1 {
int64_t& launch_counter() {
  static int64_t n = 0;
  return n;
}

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps);
std::vector<torch::Tensor> rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w,
                                       torch::Tensor rstd, c10::optional<torch::Tensor> resid);
void rope_qkv(torch::Tensor qkv, int64_t n_q, int64_t n_kv, int64_t D, torch::Tensor cos_t,
              torch::Tensor sin_t, int64_t S, bool inverse);
torch::Tensor swiglu_fwd(torch::Tensor gu);
torch::Tensor swiglu_bwd(torch::Tensor da, torch::Tensor gu);
torch::Tensor embedding_fwd(torch::Tensor ids, torch::Tensor w);
void embedding_bwd(torch::Tensor dh, torch::Tensor ids, torch::Tensor dw);
std::vector<torch::Tensor> linear_cross_entropy(torch::Tensor x, torch::Tensor w, torch::Tensor targets,
                                                torch::Tensor dx, torch::Tensor dw, int64_t chunk_rows,
                                                int64_t ignore_index);
std::vector<torch::Tensor> cross_entropy_fwd_bwd(torch::Tensor logits, torch::Tensor targets,
                                                 int64_t ignore_index, double grad_scale);
void gemm_bf16(torch::Tensor A, torch::Tensor B, torch::Tensor C, bool a_mn, bool b_mn,
               c10::optional<torch::Tensor> R);
int64_t gemm_check_error(bool reset);
void gemm_set_mode(int64_t mode);
void gemm_set_streamk(bool on);
void fused_set_peer_wait(double seconds);
int64_t gemm_get_mode();
std::vector<torch::Tensor> attention_fwd(torch::Tensor qkv, int64_t n_q, int64_t n_kv, int64_t D,
                                         int64_t S);
std::vector<torch::Tensor> attention_fwd_tc(torch::Tensor qkv, int64_t n_q, int64_t n_kv, int64_t D,
                                            int64_t S);
void attn_set_mode(int64_t mode);
void attn_fwd2_set_poly(int64_t n);
void attn_set_bwd_pipelined(bool on);
void attn_fwd2_set_debug(torch::Tensor buf);
void attn_bwd2_set_debug(torch::Tensor buf);
std::vector<torch::Tensor> attention_fwd_tc2(torch::Tensor qkv, int64_t n_q, int64_t n_kv, int64_t S);
int64_t attn_get_mode();
torch::Tensor attention_bwd(torch::Tensor dout, torch::Tensor qkv, torch::Tensor out,
                            torch::Tensor lse, int64_t n_q, int64_t n_kv, int64_t D, int64_t S);
void fused_rs_d2h(torch::Tensor ptrs, torch::Tensor sigs, int64_t rank, int64_t world,
                  int64_t offset, int64_t n, torch::Tensor host_out, double scale, int64_t epoch,
                  torch::Tensor counter, torch::Tensor err);
void fused_shard_gather(torch::Tensor ptrs, torch::Tensor sigs, int64_t rank, int64_t world,
                        int64_t offset, int64_t n, torch::Tensor host_src,
                        c10::optional<torch::Tensor> host_src_lo, int64_t epoch,
                        torch::Tensor counter, torch::Tensor err, int64_t max_ctas);
void fused_ag_qkv(torch::Tensor x, torch::Tensor unit, int64_t n_rows, torch::Tensor out,
                  torch::Tensor ptrs, torch::Tensor sigs, torch::Tensor shards, int64_t rank,
                  int64_t world, torch::Tensor host_src, c10::optional<torch::Tensor> host_src_lo,
                  int64_t epoch, torch::Tensor counters, c10::optional<torch::Tensor> rope_cos,
                  c10::optional<torch::Tensor> rope_sin, int64_t rope_S, int64_t rope_cols);
void gemm_bf16_rope(torch::Tensor A, torch::Tensor B, torch::Tensor C, torch::Tensor cos_t,
                    torch::Tensor sin_t, int64_t S, int64_t rope_cols);
void multi_tensor_adam(int64_t chunk_size, torch::Tensor noop_flag,
                       std::vector<std::vector<torch::Tensor>> tensor_lists, double lr, double beta1,
                       double beta2, double eps, int64_t step, int64_t mode, int64_t bias_correction,
                       double weight_decay);
// per-translation-unit bounds words (bounds.cuh); always 0 outside
// bounds-checked builds
unsigned long long bounds_word_attention(bool);
unsigned long long bounds_word_attention_tc(bool);
unsigned long long bounds_word_attention_fwd2(bool);
unsigned long long bounds_word_attention_bwd2(bool);
unsigned long long bounds_word_elementwise(bool);
unsigned long long bounds_word_embed_ce(bool);
unsigned long long bounds_word_fused_adam(bool);
unsigned long long bounds_word_fused_ag_gemm(bool);
unsigned long long bounds_word_fused_comm(bool);
unsigned long long bounds_word_gemm(bool);
unsigned long long bounds_word_noalloc_rmsnorm(bool);
}  // namespace t1

// [(source file, line, index)] of the first out-of-bounds access each
// kernel file recorded since the last reset; empty when none (or when the
// library was built without T1_BOUNDS_CHECK).
static std::vector<std::tuple<std::string, int64_t, int64_t>> bounds_errors(bool reset) {
  using Reader = unsigned long long (*)(bool);
  static const std::pair<const char*, Reader> readers[] = {
      {"attention.cu", &t1::bounds_word_attention},
      {"attention_tc.cu", &t1::bounds_word_attention_tc},
      {"attention_fwd2.cu", &t1::bounds_word_attention_fwd2},
      {"attention_bwd2.cu", &t1::bounds_word_attention_bwd2},
      {"elementwise.cu", &t1::bounds_word_elementwise},
      {"embed_ce.cu", &t1::bounds_word_embed_ce},
      {"fused_adam.cu", &t1::bounds_word_fused_adam},
      {"fused_ag_gemm.cu", &t1::bounds_word_fused_ag_gemm},
      {"fused_comm.cu", &t1::bounds_word_fused_comm},
      {"gemm.cu", &t1::bounds_word_gemm},
      {"noalloc_rmsnorm.cu", &t1::bounds_word_noalloc_rmsnorm},
  };
  std::vector<std::tuple<std::string, int64_t, int64_t>> out;
  for (const auto& r : readers) {
    const unsigned long long w = r.second(reset);
    if (w == ~0ull) {
      out.emplace_back(r.first, -1, -1);  // the word could not be read
    } else if (w != 0) {
      int64_t idx = static_cast<int64_t>(w & ((1ull << 40) - 1));
      if (idx & (1ll << 39)) idx -= (1ll << 40);  // sign of a negative index
      out.emplace_back(r.first, static_cast<int64_t>(w >> 40), idx);
    }
  }
  return out;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "test1_b200 sm_100a kernels";
  m.def("launch_count", [] { return t1::launch_counter(); });
#ifdef T1_BOUNDS_CHECK
  m.attr("bounds_checked") = true;
#else
  m.attr("bounds_checked") = false;
#endif
  m.def("bounds_errors", &bounds_errors, pybind11::arg("reset") = true,
        "First out-of-bounds access recorded per kernel file: [(file, line, index)]");
  m.def("clear_error", [] { return static_cast<int>(cudaGetLastError()); },
        "Return and clear the calling thread's last CUDA runtime error (e.g. after a refused "
        "cudaHostRegister that was handled)");
  m.def("rmsnorm_fwd", &t1::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &t1::rmsnorm_bwd);
  m.def("rope_qkv", &t1::rope_qkv);
  m.def("swiglu_fwd", &t1::swiglu_fwd);
  m.def("swiglu_bwd", &t1::swiglu_bwd);
  m.def("embedding_fwd", &t1::embedding_fwd);
  m.def("embedding_bwd", &t1::embedding_bwd);
  m.def("cross_entropy_fwd_bwd", &t1::cross_entropy_fwd_bwd);
  m.def("linear_cross_entropy", &t1::linear_cross_entropy,
        "chunked lm_head GEMM + cross-entropy forward/backward: (loss, count); writes dx and dW");
  m.def("gemm_bf16", &t1::gemm_bf16, pybind11::arg("A"), pybind11::arg("B"), pybind11::arg("C"),
        pybind11::arg("a_mn"), pybind11::arg("b_mn"), pybind11::arg("R") = pybind11::none());
  m.def("gemm_check_error", &t1::gemm_check_error, pybind11::arg("reset") = false);
  m.def("gemm_set_mode", &t1::gemm_set_mode, "0: single-CTA tiles, 1: CTA-pair (cta_group::2) tiles");
  m.def("fused_set_peer_wait", &t1::fused_set_peer_wait,
        "limit (seconds) of the fused NVLink kernels' waits on peer GPUs (default 60)");
  m.def("gemm_set_streamk", &t1::gemm_set_streamk, "stream-K tail of the TMA-store pair GEMM on/off");
  m.def("gemm_get_mode", &t1::gemm_get_mode);
  m.def("attention_fwd", &t1::attention_fwd);
  m.def("attention_bwd", &t1::attention_bwd);
  m.def("attention_fwd_tc", &t1::attention_fwd_tc);
  m.def("attn_set_mode", &t1::attn_set_mode,
        "0: mma.sync, 1: tcgen05 (one query tile per CTA), 2: tcgen05 forward with two query tiles per CTA");
  m.def("attn_fwd2_set_poly", &t1::attn_fwd2_set_poly);
  m.def("attn_set_bwd_pipelined", &t1::attn_set_bwd_pipelined, "tcgen05 backward: pipelined (default) or serial");
  m.def("attn_bwd2_set_debug", &t1::attn_bwd2_set_debug, "phase-stamp buffer of the pipelined backward (empty = off)");
  m.def("attn_fwd2_set_debug", &t1::attn_fwd2_set_debug, "phase-stamp buffer of the two-tile forward (empty = off)");
  m.def("attention_fwd_tc2", &t1::attention_fwd_tc2);
  m.def("attn_get_mode", &t1::attn_get_mode);
  m.def("fused_rs_d2h", &t1::fused_rs_d2h);
  m.def("fused_shard_gather", &t1::fused_shard_gather, pybind11::arg("ptrs"), pybind11::arg("sigs"),
        pybind11::arg("rank"), pybind11::arg("world"), pybind11::arg("offset"), pybind11::arg("n"),
        pybind11::arg("host_src"), pybind11::arg("host_src_lo"), pybind11::arg("epoch"),
        pybind11::arg("counter"), pybind11::arg("err"), pybind11::arg("max_ctas") = 0);
  m.def("fused_ag_qkv", &t1::fused_ag_qkv, pybind11::arg("x"), pybind11::arg("unit"),
        pybind11::arg("n_rows"), pybind11::arg("out"), pybind11::arg("ptrs"), pybind11::arg("sigs"),
        pybind11::arg("shards"), pybind11::arg("rank"), pybind11::arg("world"), pybind11::arg("host_src"),
        pybind11::arg("host_src_lo"), pybind11::arg("epoch"), pybind11::arg("counters"),
        pybind11::arg("rope_cos") = pybind11::none(), pybind11::arg("rope_sin") = pybind11::none(),
        pybind11::arg("rope_S") = 1, pybind11::arg("rope_cols") = 0);
  m.def("gemm_bf16_rope", &t1::gemm_bf16_rope,
        "C = A B^T with RoPE on columns [0, rope_cols) in the epilogue (GEMM mode 2)");
  m.def("multi_tensor_adam", &t1::multi_tensor_adam,
        "Adam/AdamW update of lists [grads, params, exp_avgs, exp_avg_sqs] (one launch per 192 tensors)");
}
