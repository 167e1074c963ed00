// Memory-bound kernels of the Llama step on sm_100a: RMSNorm forward and
// backward, rotary embedding on the fused qkv buffer, SwiGLU forward and
// backward on the fused gate/up buffer.  All move 16-byte vectors (8 bf16)
// per thread access and keep a row in registers between its passes, so each
// input byte crosses HBM once.
#include "common.cuh"

namespace t1 {

using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------- RMSNorm
// y = x * rsqrt(mean(x^2) + eps) * w, one CTA per row.
template <int VPT>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const bf16* __restrict__ x,
                                                          const bf16* __restrict__ w,
                                                          bf16* __restrict__ y,
                                                          float* __restrict__ rstd, int T, int H,
                                                          float eps) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int nvec = H >> 3;
  // uniform over the CTA: the row exists and VPT vectors per thread cover it
  if (T1_OOB(row, T) || T1_OOB(nvec - 1, VPT * (int)blockDim.x)) return;
  const bf16* xr = x + (size_t)row * H;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      load8(xr + 8 * i, v[k]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[k][j] * v[k][j];
    }
  }
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / (float)H + eps);
  bf16* yr = y + (size_t)row * H;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      float wf[8], o[8];
      load8(w + 8 * i, wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[k][j] * r * wf[j];
      store8(yr + 8 * i, o);
    }
  }
  if (threadIdx.x == 0) rstd[row] = r;
}

// dx = rstd * (dxhat - xhat * mean(dxhat * xhat)) [+ residual_grad]
// with xhat = x * rstd, dxhat = dy * w.  Each CTA walks `rows_per_cta`
// rows, keeps its columns' partial dw = sum(dy * xhat) in registers and
// writes them to dw_part[cta, :] (reduced by rmsnorm_dw_reduce_kernel).
template <int VPT>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(
    const bf16* __restrict__ dy, const bf16* __restrict__ x, const bf16* __restrict__ w,
    const float* __restrict__ rstd, const bf16* __restrict__ resid, bf16* __restrict__ dx,
    float* __restrict__ dw_part, int T, int H, int rows_per_cta) {
  __shared__ float red[32];
  const int nvec = H >> 3;
  if (T1_OOB(nvec - 1, VPT * (int)blockDim.x)) return;  // uniform over the CTA
  float wv[VPT][8], acc[VPT][8];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[k][j] = 0.f;
    if (i < nvec) load8(w + 8 * i, wv[k]);
  }
  const int r0 = blockIdx.x * rows_per_cta;
  const int r1 = min(T, r0 + rows_per_cta);
  for (int row = r0; row < r1; ++row) {
    const float r = rstd[row];
    float xh[VPT][8], dxh[VPT][8];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      int i = threadIdx.x + k * blockDim.x;
      if (i < nvec) {
        float xv[8], dv[8];
        load8(x + (size_t)row * H + 8 * i, xv);
        load8(dy + (size_t)row * H + 8 * i, dv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[k][j] = xv[j] * r;
          dxh[k][j] = dv[j] * wv[k][j];
          dot += dxh[k][j] * xh[k][j];
          acc[k][j] += dv[j] * xh[k][j];
        }
      }
    }
    dot = block_sum(dot, red);
    const float c = dot / (float)H;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      int i = threadIdx.x + k * blockDim.x;
      if (i < nvec) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = r * (dxh[k][j] - xh[k][j] * c);
        if (resid != nullptr) {
          float rv[8];
          load8(resid + (size_t)row * H + 8 * i, rv);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] += rv[j];
        }
        store8(dx + (size_t)row * H + 8 * i, o);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      float4* dst = reinterpret_cast<float4*>(dw_part + (size_t)blockIdx.x * H + 8 * i);
      dst[0] = make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]);
      dst[1] = make_float4(acc[k][4], acc[k][5], acc[k][6], acc[k][7]);
    }
  }
}

// dw[c] = sum_p dw_part[p, c] in a fixed order (deterministic).
__global__ void rmsnorm_dw_reduce_kernel(const float* __restrict__ part, int parts, int H,
                                         bf16* __restrict__ dw) {
  int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += part[(size_t)p * H + c];
  dw[c] = __float2bfloat16_rn(s);
}

// ------------------------------------------------------------------- RoPE
// In place on the q and k column blocks of qkv [T, ld]: heads 0..n_rot-1
// (n_q query heads followed by n_kv key heads), head_dim D, rotate-half
// pairs (j, j + D/2) at position t % S.  `inverse` rotates by -theta.
__global__ void rope_qkv_kernel(bf16* __restrict__ qkv, int T, int ld, int n_rot, int D,
                                const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                int S, int inverse) {
  const int half = D >> 1;
  const int per_head = half >> 3;  // 8 pairs per thread
  const long total = (long)T * n_rot * per_head;
  long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int jv = idx % per_head;
  const long th = idx / per_head;
  const int h = th % n_rot;
  const int t = th / n_rot;
  const int pos = t % S;
  if (T1_OOB((long)h * D + 8 * jv + half + 7, ld) || T1_OOB(pos, S)) return;
  bf16* base = qkv + (size_t)t * ld + (size_t)h * D + 8 * jv;
  float x1[8], x2[8];
  load8(base, x1);
  load8(base + half, x2);
  const float4* cp = reinterpret_cast<const float4*>(cos_t + (size_t)pos * half + 8 * jv);
  const float4* sp = reinterpret_cast<const float4*>(sin_t + (size_t)pos * half + 8 * jv);
  float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
  float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  float o1[8], o2[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float sj = inverse ? -s[j] : s[j];
    o1[j] = x1[j] * c[j] - x2[j] * sj;
    o2[j] = x2[j] * c[j] + x1[j] * sj;
  }
  store8(base, o1);
  store8(base + half, o2);
}

// ----------------------------------------------------------------- SwiGLU
// gu [T, 2I] = [gate | up];  a = silu(gate) * up.
__global__ void swiglu_fwd_kernel(const bf16* __restrict__ gu, bf16* __restrict__ a, int T, int I) {
  const int nv = I >> 3;
  long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)T * nv) return;
  const int t = idx / nv, v = idx % nv;
  float g[8], u[8], o[8];
  load8(gu + (size_t)t * 2 * I + 8 * v, g);
  load8(gu + (size_t)t * 2 * I + I + 8 * v, u);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = g[j] * sigmoidf_(g[j]) * u[j];
  store8(a + (size_t)t * I + 8 * v, o);
}

// dgate = da * up * s * (1 + g (1 - s)),  dup = da * g * s,  s = sigmoid(g)
__global__ void swiglu_bwd_kernel(const bf16* __restrict__ da, const bf16* __restrict__ gu,
                                  bf16* __restrict__ dgu, int T, int I) {
  const int nv = I >> 3;
  long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)T * nv) return;
  const int t = idx / nv, v = idx % nv;
  float g[8], u[8], d[8], og[8], ou[8];
  load8(gu + (size_t)t * 2 * I + 8 * v, g);
  load8(gu + (size_t)t * 2 * I + I + 8 * v, u);
  load8(da + (size_t)t * I + 8 * v, d);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float s = sigmoidf_(g[j]);
    og[j] = d[j] * u[j] * s * (1.f + g[j] * (1.f - s));
    ou[j] = d[j] * g[j] * s;
  }
  store8(dgu + (size_t)t * 2 * I + 8 * v, og);
  store8(dgu + (size_t)t * 2 * I + I + 8 * v, ou);
}

// ================================================================ host side
T1_BOUNDS_READER(elementwise)

static void check_rows(const torch::Tensor& t, int64_t H, const char* what) {
  TORCH_CHECK(t.dim() == 2 && t.size(1) == H && t.stride(1) == 1 && t.stride(0) == H, what,
              " must be a contiguous [T, ", H, "] tensor");
}

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps) {
  T1_CHECK_INPUT(x, torch::kBFloat16);
  T1_CHECK_INPUT(w, torch::kBFloat16);
  const int64_t T = x.size(0), H = x.size(1);
  check_rows(x, H, "x");
  TORCH_CHECK(w.numel() == H && w.is_contiguous(), "w must be [H]");
  TORCH_CHECK(H % 8 == 0 && H <= 16384, "hidden size must be a multiple of 8 and <= 16384");
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({T}, x.options().dtype(torch::kFloat32));
  if (T == 0) return {y, rstd};
  const int vpt = (int)((H / 8 + 255) / 256);
  const bf16* xp = (const bf16*)x.data_ptr();
  const bf16* wp = (const bf16*)w.data_ptr();
  bf16* yp = (bf16*)y.data_ptr();
  float* rp = rstd.data_ptr<float>();
  switch (vpt) {
    case 1: rmsnorm_fwd_kernel<1><<<T, 256, 0, stream()>>>(xp, wp, yp, rp, T, H, eps); break;
    case 2: rmsnorm_fwd_kernel<2><<<T, 256, 0, stream()>>>(xp, wp, yp, rp, T, H, eps); break;
    case 3:
    case 4: rmsnorm_fwd_kernel<4><<<T, 256, 0, stream()>>>(xp, wp, yp, rp, T, H, eps); break;
    default: rmsnorm_fwd_kernel<8><<<T, 256, 0, stream()>>>(xp, wp, yp, rp, T, H, eps); break;
  }
  check_launch("rmsnorm_fwd");
  count_launch();
  return {y, rstd};
}

std::vector<torch::Tensor> rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w,
                                       torch::Tensor rstd, c10::optional<torch::Tensor> resid) {
  T1_CHECK_INPUT(dy, torch::kBFloat16);
  T1_CHECK_INPUT(x, torch::kBFloat16);
  T1_CHECK_INPUT(w, torch::kBFloat16);
  T1_CHECK_INPUT(rstd, torch::kFloat32);
  const int64_t T = x.size(0), H = x.size(1);
  check_rows(x, H, "x");
  check_rows(dy, H, "dy");
  TORCH_CHECK(H % 8 == 0 && H <= 16384, "bad hidden size");
  const bf16* rp = nullptr;
  if (resid.has_value() && resid->defined()) {
    T1_CHECK_INPUT(*resid, torch::kBFloat16);
    check_rows(*resid, H, "residual_grad");
    rp = (const bf16*)resid->data_ptr();
  }
  auto dx = torch::empty_like(x);
  auto dw = torch::empty({H}, x.options());
  if (T == 0) {
    dw.zero_();
    return {dx, dw};
  }
  const int target_ctas = 2 * num_sms();
  int rows = (int)std::max<int64_t>(1, (T + target_ctas - 1) / target_ctas);
  int ctas = (int)((T + rows - 1) / rows);
  auto part = torch::empty({ctas, H}, x.options().dtype(torch::kFloat32));
  const int vpt = (int)((H / 8 + 255) / 256);
  auto* dyp = (const bf16*)dy.data_ptr();
  auto* xp = (const bf16*)x.data_ptr();
  auto* wp = (const bf16*)w.data_ptr();
  auto* rs = rstd.data_ptr<float>();
  auto* dxp = (bf16*)dx.data_ptr();
  auto* pp = part.data_ptr<float>();
  switch (vpt) {
    case 1: rmsnorm_bwd_kernel<1><<<ctas, 256, 0, stream()>>>(dyp, xp, wp, rs, rp, dxp, pp, T, H, rows); break;
    case 2: rmsnorm_bwd_kernel<2><<<ctas, 256, 0, stream()>>>(dyp, xp, wp, rs, rp, dxp, pp, T, H, rows); break;
    case 3:
    case 4: rmsnorm_bwd_kernel<4><<<ctas, 256, 0, stream()>>>(dyp, xp, wp, rs, rp, dxp, pp, T, H, rows); break;
    default: rmsnorm_bwd_kernel<8><<<ctas, 256, 0, stream()>>>(dyp, xp, wp, rs, rp, dxp, pp, T, H, rows); break;
  }
  check_launch("rmsnorm_bwd");
  rmsnorm_dw_reduce_kernel<<<(H + 255) / 256, 256, 0, stream()>>>(pp, ctas, H, (bf16*)dw.data_ptr());
  check_launch("rmsnorm_dw_reduce");
  count_launch(2);
  return {dx, dw};
}

void rope_qkv(torch::Tensor qkv, int64_t n_q, int64_t n_kv, int64_t D, torch::Tensor cos_t,
              torch::Tensor sin_t, int64_t S, bool inverse) {
  T1_CHECK_INPUT(qkv, torch::kBFloat16);
  T1_CHECK_INPUT(cos_t, torch::kFloat32);
  T1_CHECK_INPUT(sin_t, torch::kFloat32);
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1, "qkv must be row-major [T, ld]");
  TORCH_CHECK(D % 16 == 0, "head_dim must be a multiple of 16");
  TORCH_CHECK(qkv.size(1) >= (n_q + n_kv) * D, "qkv too narrow");
  TORCH_CHECK(cos_t.is_contiguous() && sin_t.is_contiguous() && cos_t.size(0) >= S &&
                  cos_t.size(1) == D / 2, "rope tables must be [>=S, D/2]");
  const int64_t T = qkv.size(0);
  TORCH_CHECK(S > 0 && T % S == 0, "tokens must be a multiple of seq_len");
  const long total = T * (n_q + n_kv) * (D / 16);
  if (total == 0) return;
  rope_qkv_kernel<<<(total + 255) / 256, 256, 0, stream()>>>(
      (bf16*)qkv.data_ptr(), T, qkv.stride(0), n_q + n_kv, D, cos_t.data_ptr<float>(),
      sin_t.data_ptr<float>(), S, inverse ? 1 : 0);
  check_launch("rope_qkv");
  count_launch();
}

torch::Tensor swiglu_fwd(torch::Tensor gu) {
  T1_CHECK_INPUT(gu, torch::kBFloat16);
  TORCH_CHECK(gu.dim() == 2 && gu.is_contiguous() && gu.size(1) % 16 == 0, "gu must be [T, 2I], I % 8 == 0");
  const int64_t T = gu.size(0), I = gu.size(1) / 2;
  auto a = torch::empty({T, I}, gu.options());
  const long total = T * (I / 8);
  if (total == 0) return a;
  swiglu_fwd_kernel<<<(total + 255) / 256, 256, 0, stream()>>>((const bf16*)gu.data_ptr(),
                                                                (bf16*)a.data_ptr(), T, I);
  check_launch("swiglu_fwd");
  count_launch();
  return a;
}

torch::Tensor swiglu_bwd(torch::Tensor da, torch::Tensor gu) {
  T1_CHECK_INPUT(da, torch::kBFloat16);
  T1_CHECK_INPUT(gu, torch::kBFloat16);
  TORCH_CHECK(gu.dim() == 2 && gu.is_contiguous() && gu.size(1) % 16 == 0, "gu must be [T, 2I]");
  const int64_t T = gu.size(0), I = gu.size(1) / 2;
  TORCH_CHECK(da.is_contiguous() && da.size(0) == T && da.size(1) == I, "da must be [T, I]");
  auto dgu = torch::empty_like(gu);
  const long total = T * (I / 8);
  if (total == 0) return dgu;
  swiglu_bwd_kernel<<<(total + 255) / 256, 256, 0, stream()>>>(
      (const bf16*)da.data_ptr(), (const bf16*)gu.data_ptr(), (bf16*)dgu.data_ptr(), T, I);
  check_launch("swiglu_bwd");
  count_launch();
  return dgu;
}

}  // namespace t1
