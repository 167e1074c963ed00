// Embedding gather / deterministic scatter-add, the fused cross-entropy
// forward + backward, and the chunked linear cross-entropy of the output
// layer on sm_100a.
#include "common.cuh"

namespace t1 {

void gemm_bf16(torch::Tensor A, torch::Tensor B, torch::Tensor C, bool a_mn, bool b_mn,
               c10::optional<torch::Tensor> R);

using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------- embedding
// h[t, :] = W[ids[t], :]
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ w,
                                     bf16* __restrict__ h, int H, int64_t V) {
  const int t = blockIdx.x;
  int64_t id = ids[t];
  if (T1_OOB(id, V)) return;      // checked builds: record and skip the row
  if (id < 0 || id >= V) id = 0;  // host-resident ids are range-checked before the copy
  const int4* src = reinterpret_cast<const int4*>(w + id * H);
  int4* dst = reinterpret_cast<int4*>(h + (size_t)t * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// dW[id, :] = sum of dh[t, :] over positions t with ids[t] == id, in
// ascending t (deterministic).  `order` is a stable sort of the positions by
// id; one CTA per sorted position, only segment heads do work.
__global__ void embedding_bwd_kernel(const int64_t* __restrict__ sorted_ids,
                                     const int64_t* __restrict__ order,
                                     const bf16* __restrict__ dh, bf16* __restrict__ dw, int T,
                                     int H, int64_t V) {
  const int i = blockIdx.x;
  const int64_t id = sorted_ids[i];
  if (T1_OOB(id, V)) return;  // checked builds: record
  if (id < 0 || id >= V) return;  // never write outside dw
  if (i > 0 && sorted_ids[i - 1] == id) return;
  int end = i + 1;
  while (end < T && sorted_ids[end] == id) ++end;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = i; j < end; ++j) {
      float v[8];
      if (T1_OOB(order[j], T)) continue;
      load8(dh + (size_t)order[j] * H + c, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += v[k];
    }
    store8(dw + id * H + c, acc);
  }
}

// ------------------------------------------------------------ cross-entropy
// count of targets != ignore_index -> *count (int), written by one CTA
__global__ void count_valid_kernel(const int64_t* __restrict__ tgt, int T, int64_t ignore,
                                   int* __restrict__ count) {
  __shared__ float red[32];
  float c = 0.f;
  for (int i = threadIdx.x; i < T; i += blockDim.x) c += tgt[i] != ignore ? 1.f : 0.f;
  c = block_sum(c, red);
  if (threadIdx.x == 0) *count = (int)c;
}

// One CTA per row of logits [T, V] (bf16, overwritten with the gradient).
// Pass 1: online max / sum-exp over the row (16-byte loads).
// Pass 2: g = (softmax - onehot(target)) * scale, written in place, where
// scale = grad_scale if > 0 else 1 / count (mean over valid targets).
// Rows whose target is ignore_index get a zero gradient and zero loss.
__global__ void __launch_bounds__(512) ce_fwd_bwd_kernel(bf16* __restrict__ logits,
                                                         const int64_t* __restrict__ tgt, int V,
                                                         int64_t ignore, float grad_scale,
                                                         const int* __restrict__ count,
                                                         float* __restrict__ row_loss) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  bf16* lr = logits + (size_t)row * V;
  const int nvec = V >> 3;
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[8];
    load8(lr + 8 * i, v);
    float vm = v[0];
#pragma unroll
    for (int k = 1; k < 8; ++k) vm = fmaxf(vm, v[k]);
    if (vm > m) {
      s *= __expf(m - vm);
      m = vm;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) s += __expf(v[k] - m);
  }
  // combine (m, s) across the block
  const float bm = block_max(m, red);
  s = (m == -INFINITY) ? 0.f : s * __expf(m - bm);
  const float bs = block_sum(s, red);
  const float lse = bm + __logf(bs);
  const int64_t t = tgt[row];
  if (t != ignore && T1_OOB(t, V)) {
  }  // checked builds: record a target that is neither ignored nor a class
  const bool valid = t != ignore && t >= 0 && t < V;
  if (threadIdx.x == 0) {
    row_loss[row] = valid ? lse - __bfloat162float(lr[t]) : 0.f;
  }
  __syncthreads();  // the target logit is read before being overwritten
  const float scale = valid ? (grad_scale > 0.f ? grad_scale : 1.f / fmaxf(1.f, (float)*count)) : 0.f;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[8];
    load8(lr + 8 * i, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float p = __expf(v[k] - lse) * scale;
      if (8 * i + k == t) p -= scale;
      v[k] = p;
    }
    store8(lr + 8 * i, v);
  }
}

// loss = sum(row_loss) / max(count, 1), one CTA, fixed order.
__global__ void ce_loss_reduce_kernel(const float* __restrict__ row_loss, int T,
                                      const int* __restrict__ count, float* __restrict__ loss) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < T; i += blockDim.x) s += row_loss[i];
  s = block_sum(s, red);
  if (threadIdx.x == 0) *loss = s / fmaxf(1.f, (float)*count);
}

// ================================================================ host side
T1_BOUNDS_READER(embed_ce)

torch::Tensor embedding_fwd(torch::Tensor ids, torch::Tensor w) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == torch::kInt64, "ids must be int64 CUDA");
  T1_CHECK_INPUT(w, torch::kBFloat16);
  TORCH_CHECK(w.dim() == 2 && w.is_contiguous() && w.size(1) % 8 == 0, "w must be [V, H], H % 8 == 0");
  auto flat = ids.reshape({-1}).contiguous();
  const int64_t T = flat.numel(), H = w.size(1);
  auto h = torch::empty({T, H}, w.options());
  if (T == 0) return h;
  embedding_fwd_kernel<<<T, 128, 0, stream()>>>(flat.data_ptr<int64_t>(), (const bf16*)w.data_ptr(),
                                                (bf16*)h.data_ptr(), H, w.size(0));
  check_launch("embedding_fwd");
  count_launch();
  return h;
}

void embedding_bwd(torch::Tensor dh, torch::Tensor ids, torch::Tensor dw) {
  T1_CHECK_INPUT(dh, torch::kBFloat16);
  T1_CHECK_INPUT(dw, torch::kBFloat16);
  TORCH_CHECK(dw.dim() == 2 && dw.is_contiguous() && dh.is_contiguous(), "bad layout");
  const int64_t H = dw.size(1);
  auto flat = ids.reshape({-1}).contiguous();
  const int64_t T = flat.numel();
  TORCH_CHECK(dh.size(0) == T && dh.size(1) == H, "dh must be [T, H]");
  T1_CHECK_CUDA(cudaMemsetAsync(dw.data_ptr(), 0, dw.numel() * 2, stream()));
  if (T == 0) return;
  auto sr = flat.sort(/*stable=*/true, 0, false);
  auto sorted = std::get<0>(sr);
  auto order = std::get<1>(sr);
  embedding_bwd_kernel<<<T, 128, 0, stream()>>>(sorted.data_ptr<int64_t>(), order.data_ptr<int64_t>(),
                                                (const bf16*)dh.data_ptr(), (bf16*)dw.data_ptr(), T, H,
                                                dw.size(0));
  check_launch("embedding_bwd");
  count_launch();
}

// Returns (loss [1] fp32 on device, count [1] int32).  logits is overwritten
// with d(loss)/d(logits) (times grad_scale if > 0).
std::vector<torch::Tensor> cross_entropy_fwd_bwd(torch::Tensor logits, torch::Tensor targets,
                                                 int64_t ignore_index, double grad_scale) {
  T1_CHECK_INPUT(logits, torch::kBFloat16);
  TORCH_CHECK(targets.is_cuda() && targets.scalar_type() == torch::kInt64, "targets must be int64 CUDA");
  TORCH_CHECK(logits.dim() == 2 && logits.is_contiguous() && logits.size(1) % 8 == 0,
              "logits must be contiguous [T, V] with V % 8 == 0");
  const int64_t T = logits.size(0), V = logits.size(1);
  TORCH_CHECK(targets.numel() == T, "targets must have T entries");
  auto tg = targets.contiguous();
  auto opts = logits.options();
  auto count = torch::empty({1}, opts.dtype(torch::kInt32));
  auto row_loss = torch::empty({T}, opts.dtype(torch::kFloat32));
  auto loss = torch::empty({1}, opts.dtype(torch::kFloat32));
  count_valid_kernel<<<1, 1024, 0, stream()>>>(tg.data_ptr<int64_t>(), T, ignore_index, count.data_ptr<int>());
  check_launch("count_valid");
  if (T > 0) {
    ce_fwd_bwd_kernel<<<T, 512, 0, stream()>>>((bf16*)logits.data_ptr(), tg.data_ptr<int64_t>(), V,
                                               ignore_index, (float)grad_scale, count.data_ptr<int>(),
                                               row_loss.data_ptr<float>());
    check_launch("ce_fwd_bwd");
  }
  ce_loss_reduce_kernel<<<1, 1024, 0, stream()>>>(row_loss.data_ptr<float>(), T, count.data_ptr<int>(),
                                                  loss.data_ptr<float>());
  check_launch("ce_loss_reduce");
  count_launch(3);
  return {loss, count};
}

// Output layer of a causal LM without the [T, V] logits: for each chunk of
// `chunk_rows` tokens, logits = x_c W^T into one reusable [chunk_rows, V]
// buffer (tcgen05 GEMM), the cross-entropy forward + backward overwrites
// them with d(loss)/d(logits) (mean over the valid targets of the WHOLE
// batch, counted once up front), then dx_c = dlogits W and
// dW (+)= dlogits^T x_c -- the first chunk stores dW, later ones add to it
// through the GEMM's residual epilogue.  Peak extra memory: chunk_rows x V
// bf16 (the reference gets the same effect from Liger's fused linear
// cross-entropy, slide_fsdp.py:86-98).  Returns (loss [1] fp32, count [1]).
std::vector<torch::Tensor> linear_cross_entropy(torch::Tensor x, torch::Tensor w, torch::Tensor targets,
                                                torch::Tensor dx, torch::Tensor dw, int64_t chunk_rows,
                                                int64_t ignore_index) {
  T1_CHECK_INPUT(x, torch::kBFloat16);
  T1_CHECK_INPUT(w, torch::kBFloat16);
  T1_CHECK_INPUT(dx, torch::kBFloat16);
  T1_CHECK_INPUT(dw, torch::kBFloat16);
  TORCH_CHECK(targets.is_cuda() && targets.scalar_type() == torch::kInt64, "targets must be int64 CUDA");
  TORCH_CHECK(x.dim() == 2 && x.is_contiguous() && w.dim() == 2 && w.is_contiguous(),
              "x [T, H] and w [V, H] must be contiguous");
  const int64_t T = x.size(0), H = x.size(1), V = w.size(0);
  TORCH_CHECK(w.size(1) == H && V % 8 == 0 && H % 8 == 0, "w must be [V, H] with V, H multiples of 8");
  TORCH_CHECK(dx.sizes() == x.sizes() && dx.is_contiguous(), "dx must be contiguous [T, H]");
  TORCH_CHECK(dw.sizes() == w.sizes() && dw.is_contiguous(), "dw must be contiguous [V, H]");
  TORCH_CHECK(targets.numel() == T, "targets must have T entries");
  TORCH_CHECK(chunk_rows > 0, "chunk_rows must be positive");
  auto tg = targets.contiguous();
  auto opts = x.options();
  auto count = torch::empty({1}, opts.dtype(torch::kInt32));
  auto row_loss = torch::empty({std::max<int64_t>(T, 1)}, opts.dtype(torch::kFloat32));
  auto loss = torch::empty({1}, opts.dtype(torch::kFloat32));
  count_valid_kernel<<<1, 1024, 0, stream()>>>(tg.data_ptr<int64_t>(), T, ignore_index, count.data_ptr<int>());
  check_launch("count_valid");
  count_launch();
  if (T == 0) {
    dw.zero_();
  } else {
    const int64_t rows_max = std::min(chunk_rows, T);
    auto buf = torch::empty({rows_max, V}, opts);
    for (int64_t t0 = 0; t0 < T; t0 += rows_max) {
      const int64_t rows = std::min(rows_max, T - t0);
      auto L = buf.narrow(0, 0, rows);
      auto xc = x.narrow(0, t0, rows);
      gemm_bf16(xc, w, L, false, false, c10::nullopt);  // logits
      ce_fwd_bwd_kernel<<<rows, 512, 0, stream()>>>((bf16*)L.data_ptr(), tg.data_ptr<int64_t>() + t0, V,
                                                     ignore_index, -1.f, count.data_ptr<int>(),
                                                     row_loss.data_ptr<float>() + t0);
      check_launch("ce_fwd_bwd (chunk)");
      count_launch();
      gemm_bf16(L, w, dx.narrow(0, t0, rows), false, true, c10::nullopt);  // dx = dlogits W
      gemm_bf16(L, xc, dw, true, true, t0 == 0 ? c10::optional<torch::Tensor>() : c10::optional<torch::Tensor>(dw));
    }
  }
  ce_loss_reduce_kernel<<<1, 1024, 0, stream()>>>(row_loss.data_ptr<float>(), T, count.data_ptr<int>(),
                                                  loss.data_ptr<float>());
  check_launch("ce_loss_reduce");
  count_launch();
  return {loss, count};
}

}  // namespace t1
