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
//               single-thread MMA issuer (P is double-buffered in shared
//               memory, so the softmax of block j+1 never waits for P_j V_j
//               unless it must rescale O):
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
constexpr int SMEM_BYTES = TILE /*Q*/ + STAGES * 2 * TILE /*K,V*/ + 2 * TILE /*P x2*/ + 1024 + 256;

struct Params {
  int S, T, n_q, n_kv, ld;  // ld: qkv row stride (elements)
  float scale_log2;         // log2(e) / sqrt(D)
  bf16* out;
  long ld_out;
  float* lse;
  int* err;
};

// 2^x with the hardware's approximate base-2 exponential (MUFU.EX2; ~2 ulp,
// flushes denormals): the softmax weights feed a bf16 operand anyway.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

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
  uint8_t* sP = sV + STAGES * TILE;  // two P buffers (block j uses j & 1)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * TILE);
  uint64_t* q_full = bars + 0;
  // K and V of a key block have their own barriers: K's stage frees as soon
  // as S = Q K^T is computed, so the next-but-one K block loads while P V of
  // the current block still holds the V stage
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [2]
  uint64_t* s_empty = bars + 11;  // [2]
  uint64_t* p_full = bars + 13;
  // p_empty[b]: P V of the last block that used P buffer b completed (so b
  // may be rewritten, and O holds every block up to that one)
  uint64_t* p_empty = bars + 14;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
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
  // uniform over the CTA, before any barrier or TMEM is set up: the
  // sequence lies inside the T rows and the heads inside the output row
  if (T1_OOB(tok0 + p.S - 1, p.T) || T1_OOB((long)p.n_q * D - 1, p.ld_out)) return;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(&p_empty[0], 1);
    mbar_init(&p_empty[1], 1);
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
        const uint32_t par = ((j >> 1) & 1) ^ 1;
        uint8_t* k = sK + st * TILE;
        uint8_t* v = sV + st * TILE;
        const int row = tok0 + j * BN;
        if (!mbar_wait(&k_empty[st], par)) {
          err.set(201);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], TILE);
        tma_load_2d(k, &tma_qkv, &k_full[st], kcol, row);
        tma_load_2d(k + BOX, &tma_qkv, &k_full[st], kcol + 64, row);
        if (!mbar_wait(&v_empty[st], par)) {
          err.set(209);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], TILE);
        tma_load_2d(v, &tma_qkv, &v_full[st], vcol, row);
        tma_load_2d(v + BOX, &tma_qkv, &v_full[st], vcol + 64, row);
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
        if (!mbar_wait(&k_full[st], (j >> 1) & 1)) { err.set(203); return false; }
        if (!mbar_wait(&s_empty[st], ((j >> 1) & 1) ^ 1)) { err.set(204); return false; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * TILE);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          mma_bf16(t_s0 + st * BN, kmajor_desc(q_addr, k), kmajor_desc(k_addr, k), IDESC_S, k != 0);
        mma_commit(&s_full[st]);
        mma_commit(&k_empty[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_blocks && !*abort_flag; ++j) {
        if (j + 1 < n_blocks && !issue_s(j + 1)) { ok = false; break; }
        // O += P_j V_j once the softmax warps published P_j (and rescaled O)
        if (!mbar_wait(p_full, j & 1)) { err.set(205); ok = false; break; }
        if (!mbar_wait(&v_full[j & 1], (j >> 1) & 1)) { err.set(210); ok = false; break; }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + (j & 1) * TILE);
        const uint32_t pj_addr = p_addr + (j & 1) * TILE;
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          // V block: 128 keys (the K extent) x 128 dims in two 64-dim boxes
          const uint64_t vd = smem_desc_sw128(v_addr + k * 2048, BOX, 1024);
          mma_bf16(t_o, kmajor_desc(pj_addr, k), vd, IDESC_O, (j | k) != 0);
        }
        mma_commit(&v_empty[j & 1]);
        mma_commit(&p_empty[j & 1]);
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
      // raw scores of this row: 4 chunks of 32 columns, all loads in flight
      // before the one wait (one warp per scheduler: latency is the cost)
      float sv[BN];
      {
        uint32_t u[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(t_s0 + st * BN + lane_base + c * 32, u[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(u[c][i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[st]);
      // causal mask: only the diagonal block and a block crossing the
      // sequence end need it (every other key precedes every query here)
      const int kbase = j * BN;
      if (kbase + BN - 1 > q0 || kbase + BN > p.S) {
#pragma unroll
        for (int i = 0; i < BN; ++i) {
          const int kpos = kbase + i;
          if (kpos > qpos || kpos >= p.S) sv[i] = -INFINITY;
        }
      }
      // row maximum: 8 independent chains, then combined (a single chain of
      // 128 dependent max operations would stall on latency)
      float mxs[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mxs[k] = sv[k];
#pragma unroll
      for (int i = 8; i < BN; ++i) mxs[i & 7] = fmaxf(mxs[i & 7], sv[i]);
      float mx = fmaxf(fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3])),
                       fmaxf(fmaxf(mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7])));
      mx *= p.scale_log2;
      // Lazy rescaling: the exponent base m moves only when this block's
      // maximum exceeds it by more than 8 (a factor 256), so most blocks
      // skip the O rescale; p = 2^(s - m) then stays below 256, far inside
      // fp32 and bf16 range, and O / l and the LSE use the same m.
      float alpha = 1.f;
      if (__any_sync(0xffffffffu, mx > m + 8.f)) {
        const float m_new = fmaxf(m, mx);
        alpha = (m == -INFINITY) ? 0.f : ex2_approx(m - m_new);
        m = m_new;
      }
      const float mb = (m == -INFINITY) ? 0.f : m;
      float sums[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < BN; ++i) {
        const float e = ex2_approx(fmaf(sv[i], p.scale_log2, -mb));
        sv[i] = e;
        sums[i & 7] += e;
      }
      const float sum = ((sums[0] + sums[1]) + (sums[2] + sums[3])) + ((sums[4] + sums[5]) + (sums[6] + sums[7]));
      l = l * alpha + sum;
      // P buffer j & 1 is free once P_{j-2} V_{j-2} completed (its
      // (j >> 1)-th use); with the other buffer P_{j-1} V_{j-1} may still run
      if (j > 1) {
        int w2 = 0;
        if (lane == 0) w2 = !*abort_flag && mbar_wait(&p_empty[j & 1], ((j >> 1) - 1) & 1);
        if (!__shfl_sync(0xffffffffu, w2, 0)) {
          if (lane == 0 && !*abort_flag) { err.set(207); *abort_flag = 1; }
          ok = false;
          break;
        }
      }
      // P (bf16) into the 128B-swizzled K-major layout: row r, 16 chunks of
      // 8 keys; chunk u of a 64-key box sits at unit (u ^ (r & 7))
      uint8_t* pbuf = sP + (j & 1) * TILE;
#pragma unroll
      for (int c16 = 0; c16 < BN / 8; ++c16) {
        uint4 pk;
        __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
        for (int t = 0; t < 4; ++t) h2[t] = __floats2bfloat162_rn(sv[c16 * 8 + 2 * t], sv[c16 * 8 + 2 * t + 1]);
        const int box = c16 >> 3, u = c16 & 7;
        *reinterpret_cast<uint4*>(pbuf + box * BOX + r * 128 + ((u ^ (r & 7)) << 4)) = pk;
      }
      fence_proxy_async_smem();
      // rescale O when this warp moved its exponent base (alpha == 1
      // otherwise); O must first hold every block before j: P_{j-1} V_{j-1}
      // is the ((j - 1) >> 1)-th completion of p_empty[(j - 1) & 1]
      const bool rescale = j > 0 && __any_sync(0xffffffffu, alpha != 1.f);
      if (rescale) {
        int w3 = 0;
        if (lane == 0) w3 = !*abort_flag && mbar_wait(&p_empty[(j - 1) & 1], ((j - 1) >> 1) & 1);
        if (!__shfl_sync(0xffffffffu, w3, 0)) {
          if (lane == 0 && !*abort_flag) { err.set(211); *abort_flag = 1; }
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (rescale) {
        uint32_t u[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(t_o + lane_base + c * 32, u[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int i = 0; i < 32; ++i) u[c][i] = __float_as_uint(__uint_as_float(u[c][i]) * alpha);
          tmem_st_32x32b_x32(t_o + lane_base + c * 32, u[c]);
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
      if (lane == 0) w = !*abort_flag && mbar_wait(&p_empty[(n_blocks - 1) & 1], ((n_blocks - 1) >> 1) & 1);
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


// ------------------------------------------------------------------ backward
// One CTA per (128-key block, KV head, sequence); it loops over the query
// heads of its group and the query blocks at or after its key block.  TMEM
// (512 columns): S | dP | dK | dV, 128 columns each; dQ of a query block
// reuses the S columns once P and dS are in shared memory.
//   MMA1:  S = Q K^T, dP = dO V^T
//   warps 2-5 (thread r = query row): P = exp2(S*scale*log2e - lse*log2e)
//          (causal mask), dS = P (dP - delta); P and dS -> shared memory
//   MMA2:  dV += P^T dO, dK += dS^T Q, dQ = dS K
//   warps 2-5: dQ * scale -> fp32 global accumulation (vector atomics);
//          after the last block, dK * scale and dV -> bf16 dqkv.
// Q/dO are single-buffered: the next pair is loaded while the softmax warps
// drain dQ.
constexpr int BWD_SMEM_BYTES = 6 * TILE + 1024 + 256;

struct BwdParams {
  int S, T, n_q, n_kv;
  float scale, scale_log2;
  const float* lse;    // [Hq, T], natural log
  const float* delta;  // [Hq, T]
  float* dq_acc;       // [T, Hq, D]
  bf16* dqkv;
  long ldd;
  int* err;
};

// MN-major operand tile: 128 rows of the K extent, 128 MN columns in two
// 64-column boxes; descriptor of k-step k (16 rows).
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int k) {
  return smem_desc_sw128(base + k * 2048, BOX, 1024);
}

__global__ void __launch_bounds__(192, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tma_qkv,
                       const __grid_constant__ CUtensorMap tma_do, const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + TILE;
  uint8_t* sQ = sV + TILE;
  uint8_t* sDO = sQ + TILE;
  uint8_t* sP = sDO + TILE;
  uint8_t* sDS = sP + TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDS + TILE);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;
  uint64_t* s_full = bars + 2;
  uint64_t* pds_full = bars + 3;
  uint64_t* mma2_done = bars + 4;
  uint64_t* s_free = bars + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const ErrorSlot err{p.err};
  const int kb = blockIdx.x;  // heavy (early) key blocks first
  const int g = blockIdx.y;
  const int b = blockIdx.z;
  const int G = p.n_q / p.n_kv;
  const int tok0 = b * p.S;
  const int nqb = (p.S + BM - 1) / BM;
  const int per_head = nqb - kb;
  const int n_it = G * per_head;
  // uniform over the CTA, before any barrier or TMEM is set up
  if (T1_OOB(tok0 + p.S - 1, p.T) || T1_OOB((long)(p.n_q + 2 * p.n_kv) * D - 1, p.ldd) ||
      T1_OOB(kb, nqb))
    return;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(qdo_full, 1);
    mbar_init(s_full, 1);
    mbar_init(pds_full, 4);
    mbar_init(mma2_done, 1);
    mbar_init(s_free, 4);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tma_qkv);
    prefetch_tensormap(&tma_do);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dk = tmem + 256, t_dv = tmem + 384;

  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (lane == 0) {
      const int kcol = (p.n_q + g) * D, vcol = (p.n_q + p.n_kv + g) * D;
      const int krow = tok0 + kb * BN;
      mbar_arrive_expect_tx(kv_full, 2 * TILE);
      tma_load_2d(sK, &tma_qkv, kv_full, kcol, krow);
      tma_load_2d(sK + BOX, &tma_qkv, kv_full, kcol + 64, krow);
      tma_load_2d(sV, &tma_qkv, kv_full, vcol, krow);
      tma_load_2d(sV + BOX, &tma_qkv, kv_full, vcol + 64, krow);
      for (int it = 0; it < n_it && !*abort_flag; ++it) {
        const int h = g * G + it / per_head;
        const int qb = kb + it % per_head;
        if (it > 0 && !mbar_wait(mma2_done, (it - 1) & 1)) {
          err.set(221);
          *abort_flag = 1;
          break;
        }
        const int qrow = tok0 + qb * BM;
        mbar_arrive_expect_tx(qdo_full, 2 * TILE);
        tma_load_2d(sQ, &tma_qkv, qdo_full, h * D, qrow);
        tma_load_2d(sQ + BOX, &tma_qkv, qdo_full, h * D + 64, qrow);
        tma_load_2d(sDO, &tma_do, qdo_full, h * D, qrow);
        tma_load_2d(sDO + BOX, &tma_do, qdo_full, h * D + 64, qrow);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_KK = idesc_bf16_f32(BM, BN, false, false);  // S, dP
      constexpr uint32_t ID_MM = idesc_bf16_f32(BN, D, true, true);     // dV, dK
      constexpr uint32_t ID_KM = idesc_bf16_f32(BM, D, false, true);    // dQ
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), q_addr = smem_u32(sQ);
      const uint32_t do_addr = smem_u32(sDO), p_addr = smem_u32(sP), ds_addr = smem_u32(sDS);
      bool ok = mbar_wait(kv_full, 0);
      if (!ok) err.set(222);
      for (int it = 0; ok && it < n_it && !*abort_flag; ++it) {
        if (!mbar_wait(qdo_full, it & 1)) { err.set(223); ok = false; break; }
        if (it > 0 && !mbar_wait(s_free, (it - 1) & 1)) { err.set(224); ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          mma_bf16(t_s, kmajor_desc(q_addr, k), kmajor_desc(k_addr, k), ID_KK, k != 0);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          mma_bf16(t_dp, kmajor_desc(do_addr, k), kmajor_desc(v_addr, k), ID_KK, k != 0);
        mma_commit(s_full);
        if (!mbar_wait(pds_full, it & 1)) { err.set(225); ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < BM / 16; ++k)
          mma_bf16(t_dv, mnmajor_desc(p_addr, k), mnmajor_desc(do_addr, k), ID_MM, (it | k) != 0);
#pragma unroll
        for (int k = 0; k < BM / 16; ++k)
          mma_bf16(t_dk, mnmajor_desc(ds_addr, k), mnmajor_desc(q_addr, k), ID_MM, (it | k) != 0);
#pragma unroll
        for (int k = 0; k < BN / 16; ++k)
          mma_bf16(t_s, kmajor_desc(ds_addr, k), mnmajor_desc(k_addr, k), ID_KM, k != 0);
        mma_commit(mma2_done);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // --------------------------------------------- softmax / dQ / dK dV warps
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;
    // warp-uniform bounded wait
    auto wait_w = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
      int w = 0;
      if (lane == 0) {
        w = !*abort_flag && mbar_wait(bar, parity);
        if (!w && !*abort_flag) {
          err.set(code);
          *abort_flag = 1;
        }
      }
      return __shfl_sync(0xffffffffu, w, 0) != 0;
    };
    // dQ of iteration `it` (in the S columns) -> global accumulation
    auto drain_dq = [&](int it) {
      const int h = g * G + it / per_head;
      const int qpos = (kb + it % per_head) * BM + r;
      float* dst = p.dq_acc + (static_cast<long>(tok0 + qpos) * p.n_q + h) * D;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(t_s + lane_base + c * 32, u);
        tmem_ld_wait();
        if (qpos < p.S) {
#pragma unroll
          for (int v = 0; v < 8; ++v)
            atomicAdd(reinterpret_cast<float4*>(dst + c * 32 + 4 * v),
                      make_float4(__uint_as_float(u[4 * v]) * p.scale, __uint_as_float(u[4 * v + 1]) * p.scale,
                                  __uint_as_float(u[4 * v + 2]) * p.scale, __uint_as_float(u[4 * v + 3]) * p.scale));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
    };
    for (int it = 0; it < n_it; ++it) {
      const int h = g * G + it / per_head;
      const int qb = kb + it % per_head;
      const int qpos = qb * BM + r;
      const bool q_ok = qpos < p.S;
      const float lse2 = q_ok ? p.lse[static_cast<long>(h) * p.T + tok0 + qpos] * LOG2E : 0.f;
      const float dlt = q_ok ? p.delta[static_cast<long>(h) * p.T + tok0 + qpos] : 0.f;
      if (it > 0) {
        // MMA2 of it-1 done: dQ(it-1) ready, P/dS buffers free
        if (!wait_w(mma2_done, (it - 1) & 1, 226)) { ok = false; break; }
        tc_fence_after();
        drain_dq(it - 1);
      }
      if (!wait_w(s_full, it & 1, 227)) { ok = false; break; }
      tc_fence_after();
      const int kbase = kb * BN;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t us[32], ud[32];
        tmem_ld_32x32b_x32(t_s + lane_base + c * 32, us);
        tmem_ld_32x32b_x32(t_dp + lane_base + c * 32, ud);
        tmem_ld_wait();
        float pv[32], dsv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int kpos = kbase + c * 32 + i;
          const float pe = (q_ok && kpos <= qpos) ? ex2_approx(fmaf(__uint_as_float(us[i]), p.scale_log2, -lse2))
                                                  : 0.f;
          pv[i] = pe;
          dsv[i] = pe * (__uint_as_float(ud[i]) - dlt);
        }
        // 32 keys = 4 units of 8 in box c >> 1, units (c & 1) * 4 .. + 3
#pragma unroll
        for (int u8 = 0; u8 < 4; ++u8) {
          uint4 pk, dk;
          __nv_bfloat162* hp = reinterpret_cast<__nv_bfloat162*>(&pk);
          __nv_bfloat162* hd = reinterpret_cast<__nv_bfloat162*>(&dk);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            hp[t] = __floats2bfloat162_rn(pv[u8 * 8 + 2 * t], pv[u8 * 8 + 2 * t + 1]);
            hd[t] = __floats2bfloat162_rn(dsv[u8 * 8 + 2 * t], dsv[u8 * 8 + 2 * t + 1]);
          }
          const int unit = (c & 1) * 4 + u8;
          const uint32_t off = (c >> 1) * BOX + r * 128 + ((unit ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(sP + off) = pk;
          *reinterpret_cast<uint4*>(sDS + off) = dk;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pds_full);
    }
    if (ok && n_it > 0) {
      if (wait_w(mma2_done, (n_it - 1) & 1, 228)) {
        tc_fence_after();
        drain_dq(n_it - 1);
        // dK (scaled) and dV rows: TMEM lane r = key row r of the block.  All
        // lanes load (the TMEM loads are warp-collective); only valid rows store.
        const int kpos = kb * BN + r;
        const bool k_ok = kpos < p.S;
        bf16* dk_row = p.dqkv + static_cast<long>(tok0 + kpos) * p.ldd + (p.n_q + g) * D;
        bf16* dv_row = p.dqkv + static_cast<long>(tok0 + kpos) * p.ldd + (p.n_q + p.n_kv + g) * D;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t uk[32], uv[32];
          tmem_ld_32x32b_x32(t_dk + lane_base + c * 32, uk);
          tmem_ld_32x32b_x32(t_dv + lane_base + c * 32, uv);
          tmem_ld_wait();
          if (k_ok) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 a, bq;
              __nv_bfloat162* ha = reinterpret_cast<__nv_bfloat162*>(&a);
              __nv_bfloat162* hb = reinterpret_cast<__nv_bfloat162*>(&bq);
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                ha[t] = __floats2bfloat162_rn(__uint_as_float(uk[v * 8 + 2 * t]) * p.scale,
                                              __uint_as_float(uk[v * 8 + 2 * t + 1]) * p.scale);
                hb[t] = __floats2bfloat162_rn(__uint_as_float(uv[v * 8 + 2 * t]),
                                              __uint_as_float(uv[v * 8 + 2 * t + 1]));
              }
              *reinterpret_cast<uint4*>(dk_row + c * 32 + v * 8) = a;
              *reinterpret_cast<uint4*>(dv_row + c * 32 + v * 8) = bq;
            }
          }
        }
      }
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

T1_BOUNDS_READER(attention_tc)


// Backward core (tcgen05): writes dK/dV into dqkv and accumulates scaled dQ
// into dq_acc [T, Hq, D] fp32 (zeroed by the caller); delta = rowsum(dO * O).
void attention_bwd_tc_core(torch::Tensor dout, torch::Tensor qkv, torch::Tensor lse,
                           torch::Tensor delta, torch::Tensor dq_acc, torch::Tensor dqkv, int64_t n_q,
                           int64_t n_kv, int64_t S) {
  const int64_t T = qkv.size(0), B = T / S;
  const CUtensorMap mq = make_map(qkv.data_ptr(), qkv.size(1), T, qkv.stride(0), 128);
  const CUtensorMap md = make_map(dout.data_ptr(), dout.size(1), T, dout.stride(0), 128);
  attn_tc::BwdParams p;
  p.S = static_cast<int>(S);
  p.T = static_cast<int>(T);
  p.n_q = static_cast<int>(n_q);
  p.n_kv = static_cast<int>(n_kv);
  p.scale = 1.0f / std::sqrt(static_cast<float>(attn_tc::D));
  p.scale_log2 = p.scale * attn_tc::LOG2E;
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  p.ldd = dqkv.stride(0);
  p.err = gemm_error_word().data_ptr<int>();
  static bool cfg = false;
  if (!cfg) {
    T1_CHECK_CUDA(cudaFuncSetAttribute(attn_tc::attn_bwd_tc_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, attn_tc::BWD_SMEM_BYTES));
    cfg = true;
  }
  dim3 grid((S + attn_tc::BN - 1) / attn_tc::BN, n_kv, B);
  attn_tc::attn_bwd_tc_kernel<<<grid, 192, attn_tc::BWD_SMEM_BYTES, stream()>>>(mq, md, p);
  check_launch("attention_bwd_tc");
  count_launch();
}

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
