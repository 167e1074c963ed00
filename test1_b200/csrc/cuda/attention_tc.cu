// Causal GQA attention forward on the 5th-generation tensor cores
// (tcgen05), head_dim 128, on the fused qkv buffer [T, (Hq + 2 Hkv) * 128].
// Same outputs as the mma.sync kernel in attention.cu (o [T, Hq*128] bf16,
// lse [Hq, T] natural log with the 1/sqrt(d) scale included), so the
// backward kernels consume either.
//
// One CTA per (128-query block, head, sequence); 192 threads:
//   warp 0      TMA producer: Q once (2 x 64-column boxes), then K and V of
//               each 128-key block into a 2-stage ring (no multicast)
//   warp 1      TMEM owner (384 of 512 columns: S double buffer + O) and
//               single-thread MMA issuer:
//                 S[j%2] = Q K_j^T        (M 128, N 128, K 128; A, B K-major)
//                 O     += P_j V_j        (M 128, N 128, K 128; P K-major
//                                          from shared memory, V MN-major)
//               S of block j+1 is issued before P_j V_j, so the tensor core
//               computes the next scores while the softmax warps work
//   warps 2-5   softmax: thread r owns query row r (its TMEM lane): reads
//               S, applies scale and the causal mask, keeps the running max
//               and sum in base 2, writes P (bf16) into the 128B-swizzled
//               shared-memory layout the MMA descriptor reads, rescales O in
//               TMEM when a warp's maximum moved, and finally writes
//               O / l and the log-sum-exp.
// Every wait is bounded (sm100.cuh); a timeout writes the error word.
#include "common.cuh"
#include "sm100.cuh"

namespace t1 {

CUtensorMap make_map(const void* ptr, int64_t inner, int64_t outer, int64_t ld, int box_outer);
torch::Tensor& gemm_error_word();

namespace attn_tc {

using namespace sm100;
using bf16 = __nv_bfloat16;

constexpr int D = 128;
constexpr int BM = 128;           // query rows per CTA
constexpr int BN = 128;           // keys per block
constexpr int BOX = 128 * 64 * 2;  // one 128-row x 64-column bf16 box: 16 KB
constexpr int TILE = 2 * BOX;      // 128 x 128 bf16 (two boxes): 32 KB
constexpr int STAGES = 2;
constexpr float LOG2E = 1.4426950408889634f;
constexpr int SMEM_BYTES = TILE /*Q*/ + STAGES * 2 * TILE /*K,V*/ + TILE /*P*/ + 1024 + 256;

struct Params {
  int S, T, n_q, n_kv, ld;  // ld: qkv row stride (elements)
  float scale_log2;         // log2(e) / sqrt(D)
  bf16* out;
  long ld_out;
  float* lse;
  int* err;
};

// K-major 128-row operand made of two 64-column swizzled boxes: descriptor
// of k-step k (16 columns) of the 128-column extent.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int k) {
  return smem_desc_sw128(base + (k >> 2) * BOX + (k & 3) * 32, 16, 1024);
}

__global__ void __launch_bounds__(192, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tma_qkv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + TILE;
  uint8_t* sV = sK + STAGES * TILE;
  uint8_t* sP = sV + STAGES * TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + TILE);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_empty = bars + 7;   // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* pv_done = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const ErrorSlot err{p.err};
  // heavy (late) query blocks first
  const int qb = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int g = h / (p.n_q / p.n_kv);
  const int tok0 = b * p.S;
  const int q0 = qb * BM;                       // first query position of this block
  const int n_blocks = min(qb + 1, (p.S + BN - 1) / BN);  // causal: key blocks 0..qb

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) prefetch_tensormap(&tma_qkv);
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s0 = tmem;        // S buffers: columns [0, 128), [128, 256)
  const uint32_t t_o = tmem + 256;   // O: columns [256, 384)

  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (lane == 0) {
      const int qcol = h * D, kcol = (p.n_q + g) * D, vcol = (p.n_q + p.n_kv + g) * D;
      mbar_arrive_expect_tx(q_full, TILE);
      tma_load_2d(sQ, &tma_qkv, q_full, qcol, tok0 + q0);
      tma_load_2d(sQ + BOX, &tma_qkv, q_full, qcol + 64, tok0 + q0);
      for (int j = 0; j < n_blocks && !*abort_flag; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1)) {
          err.set(201);
          *abort_flag = 1;
          break;
        }
        uint8_t* k = sK + st * TILE;
        uint8_t* v = sV + st * TILE;
        const int row = tok0 + j * BN;
        mbar_arrive_expect_tx(&kv_full[st], 2 * TILE);
        tma_load_2d(k, &tma_qkv, &kv_full[st], kcol, row);
        tma_load_2d(k + BOX, &tma_qkv, &kv_full[st], kcol + 64, row);
        tma_load_2d(v, &tma_qkv, &kv_full[st], vcol, row);
        tma_load_2d(v + BOX, &tma_qkv, &kv_full[st], vcol + 64, row);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BN, false, false);
      constexpr uint32_t IDESC_O = idesc_bf16_f32(BM, D, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t p_addr = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0);
      if (!ok) err.set(202);
      // S(j) = Q K_j^T into S buffer j%2
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&kv_full[st], (j >> 1) & 1)) { err.set(203); return false; }
        if (!mbar_wait(&s_empty[st], ((j >> 1) & 1) ^ 1)) { err.set(204); return false; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * TILE);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          mma_bf16(t_s0 + st * BN, kmajor_desc(q_addr, k), kmajor_desc(k_addr, k), IDESC_S, k != 0);
        mma_commit(&s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_blocks && !*abort_flag; ++j) {
        if (j + 1 < n_blocks && !issue_s(j + 1)) { ok = false; break; }
        // O += P_j V_j once the softmax warps published P_j (and rescaled O)
        if (!mbar_wait(p_full, j & 1)) { err.set(205); ok = false; break; }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + (j & 1) * TILE);
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          // V block: 128 keys (the K extent) x 128 dims in two 64-dim boxes
          const uint64_t vd = smem_desc_sw128(v_addr + k * 2048, BOX, 1024);
          mma_bf16(t_o, kmajor_desc(p_addr, k), vd, IDESC_O, (j | k) != 0);
        }
        mma_commit(&kv_empty[j & 1]);
        mma_commit(pv_done);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------------ softmax warps
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;        // query row within the block == TMEM lane
    const int qpos = q0 + r;                  // query position in the sequence
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    float m = -INFINITY;  // running max (base 2, scale included)
    float l = 0.f;        // running sum
    bool ok = true;
    for (int j = 0; j < n_blocks; ++j) {
      const int st = j & 1;
      int w = 0;
      if (lane == 0) w = !*abort_flag && mbar_wait(&s_full[st], (j >> 1) & 1);
      if (!__shfl_sync(0xffffffffu, w, 0)) {
        if (lane == 0 && !*abort_flag) { err.set(206); *abort_flag = 1; }
        ok = false;
        break;
      }
      tc_fence_after();
      // scores of this row: 4 chunks of 32 columns
      float sv[BN];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(t_s0 + st * BN + lane_base + c * 32, u);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(u[i]) * p.scale_log2;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[st]);
      // causal mask (diagonal block) and keys past the sequence end
      const int kbase = j * BN;
      float mx = m;
#pragma unroll
      for (int i = 0; i < BN; ++i) {
        const int kpos = kbase + i;
        if (kpos > qpos || kpos >= p.S) sv[i] = -INFINITY;
        mx = fmaxf(mx, sv[i]);
      }
      const float alpha = (mx == -INFINITY) ? 1.f : exp2f(m - mx);
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < BN; ++i) {
        const float e = (mx == -INFINITY) ? 0.f : exp2f(sv[i] - mx);
        sv[i] = e;
        sum += e;
      }
      l = l * alpha + sum;
      m = mx;
      // P_j may overwrite the P buffer once P_{j-1} V_{j-1} completed; that
      // completion also makes O hold every block before j
      if (j > 0) {
        int w2 = 0;
        if (lane == 0) w2 = !*abort_flag && mbar_wait(pv_done, (j - 1) & 1);
        if (!__shfl_sync(0xffffffffu, w2, 0)) {
          if (lane == 0 && !*abort_flag) { err.set(207); *abort_flag = 1; }
          ok = false;
          break;
        }
        tc_fence_after();
      }
      // P (bf16) into the 128B-swizzled K-major layout: row r, 16 chunks of
      // 8 keys; chunk u of a 64-key box sits at unit (u ^ (r & 7))
#pragma unroll
      for (int c16 = 0; c16 < BN / 8; ++c16) {
        uint4 pk;
        __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
        for (int t = 0; t < 4; ++t) h2[t] = __floats2bfloat162_rn(sv[c16 * 8 + 2 * t], sv[c16 * 8 + 2 * t + 1]);
        const int box = c16 >> 3, u = c16 & 7;
        *reinterpret_cast<uint4*>(sP + box * BOX + r * 128 + ((u ^ (r & 7)) << 4)) = pk;
      }
      fence_proxy_async_smem();
      // rescale O when this warp's maximum moved (alpha == 1 otherwise)
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t u[32];
          tmem_ld_32x32b_x32(t_o + lane_base + c * 32, u);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * alpha);
          tmem_st_32x32b_x32(t_o + lane_base + c * 32, u);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // epilogue: wait for the last P V, normalise, store O and the LSE
    if (ok) {
      int w = 0;
      if (lane == 0) w = !*abort_flag && mbar_wait(pv_done, (n_blocks - 1) & 1);
      if (!__shfl_sync(0xffffffffu, w, 0)) {
        if (lane == 0 && !*abort_flag) { err.set(208); *abort_flag = 1; }
        ok = false;
      }
    }
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool row_ok = qpos < p.S;
      bf16* orow = p.out + static_cast<long>(tok0 + qpos) * p.ld_out + h * D;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(t_o + lane_base + c * 32, u);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 pk;
            __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
            for (int t = 0; t < 4; ++t)
              h2[t] = __floats2bfloat162_rn(__uint_as_float(u[v * 8 + 2 * t]) * inv,
                                            __uint_as_float(u[v * 8 + 2 * t + 1]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + v * 8) = pk;
          }
        }
      }
      if (row_ok) p.lse[static_cast<long>(h) * p.T + tok0 + qpos] = (m + log2f(l)) / LOG2E;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn_tc

std::vector<torch::Tensor> attention_fwd_tc(torch::Tensor qkv, int64_t n_q, int64_t n_kv, int64_t D,
                                            int64_t S) {
  T1_CHECK_INPUT(qkv, torch::kBFloat16);
  TORCH_CHECK(D == attn_tc::D, "attention kernels are built for head_dim 128, got ", D);
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.size(1) >= (n_q + 2 * n_kv) * D,
              "qkv must be row-major [T, (n_q + 2 n_kv) D]");
  TORCH_CHECK(n_q % n_kv == 0, "n_q must be a multiple of n_kv");
  TORCH_CHECK(S % 64 == 0 && qkv.size(0) % S == 0, "seq_len must be a multiple of 64 and divide T");
  const int64_t T = qkv.size(0), B = T / S;
  auto out = torch::empty({T, n_q * D}, qkv.options());
  auto lse = torch::empty({n_q, T}, qkv.options().dtype(torch::kFloat32));
  const CUtensorMap map = make_map(qkv.data_ptr(), qkv.size(1), T, qkv.stride(0), 128);
  attn_tc::Params p;
  p.S = static_cast<int>(S);
  p.T = static_cast<int>(T);
  p.n_q = static_cast<int>(n_q);
  p.n_kv = static_cast<int>(n_kv);
  p.ld = static_cast<int>(qkv.stride(0));
  p.scale_log2 = attn_tc::LOG2E / std::sqrt(static_cast<float>(D));
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ld_out = out.stride(0);
  p.lse = lse.data_ptr<float>();
  p.err = gemm_error_word().data_ptr<int>();
  static bool cfg = false;
  if (!cfg) {
    T1_CHECK_CUDA(cudaFuncSetAttribute(attn_tc::attn_fwd_tc_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, attn_tc::SMEM_BYTES));
    cfg = true;
  }
  dim3 grid((S + attn_tc::BM - 1) / attn_tc::BM, n_q, B);
  attn_tc::attn_fwd_tc_kernel<<<grid, 192, attn_tc::SMEM_BYTES, stream()>>>(map, p);
  check_launch("attention_fwd_tc");
  count_launch();
  return {out, lse};
}

}  // namespace t1
