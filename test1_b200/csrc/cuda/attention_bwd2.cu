// Causal GQA attention backward on tcgen05, pipelined (head_dim 128, fused
// qkv layout).  Same contract as attn_bwd_tc_kernel (attention_tc.cu): dK and
// dV (bf16) into dqkv, dQ * scale accumulated into dq_acc [T, Hq, D] fp32
// (zeroed by the caller), delta = rowsum(dO * O) precomputed.
//
// One CTA per (128-key block, KV head, sequence), looping over the query
// heads of its group and the query blocks at or after its key block.
// TMEM (512 columns): S | dP | dK | dV.  Per iteration `it`:
//   MMA  S = Q K^T, dP = dO V^T             (commit s_full)
//   softmax warps: P = exp2(S*scale*log2e - lse*log2e) (causal mask),
//        dS = P (dP - delta) -> shared memory  (arrive pds_full)
//   MMA  dV += P^T dO   (commit do_free: dO's buffer may be reloaded)
//        dQ  = dS K     into the dP columns (commit dq_ready)
//        dK += dS^T Q   (commit q_free of Q's buffer)
//   softmax warps: dQ * scale -> fp32 global accumulation (TMA bulk
//        reduce-adds of 32 x 32 boxes staged in shared memory), arriving
//        dq_free as soon as the dP columns are read
// What overlaps: Q is double-buffered and loaded ahead; dO is reloaded as
// soon as dV has read it (while dQ and dK run); S of the next iteration is
// computed while the softmax warps drain dQ, and the next dP as soon as the
// drain finished.  The tensor core then waits only for the softmax pass.
// Warps: 0 TMA producer, 1 TMEM owner + MMA issuer, 2-5 softmax / drain /
// epilogue.  Every wait is bounded (sm100.cuh); a timeout writes the error
// word.  No TMA load uses multicast.
#include "common.cuh"
#include "sm100.cuh"

namespace t1 {

CUtensorMap make_map(const void* ptr, int64_t inner, int64_t outer, int64_t ld, int box_outer);
CUtensorMap make_map_f32(const void* ptr, int64_t inner, int64_t outer, int64_t ld);
torch::Tensor& gemm_error_word();

namespace attn_bwd2 {

using namespace sm100;
using bf16 = __nv_bfloat16;

constexpr int D = 128;
constexpr int BM = 128;            // query rows per iteration
constexpr int BN = 128;            // keys per CTA
constexpr int BOX = 128 * 64 * 2;  // 128 rows x 64 columns bf16
constexpr int TILE = 2 * BOX;      // 128 x 128 bf16
constexpr float LOG2E = 1.4426950408889634f;
// K, V, Q[2], dO, P, dS
constexpr int SMEM_BYTES = 7 * TILE + 1024 + 256;
static_assert(SMEM_BYTES <= 232448, "pipelined attention backward exceeds 227 KB of shared memory");

struct Params {
  int S, T, n_q, n_kv;
  float scale, scale_log2;
  const float* lse;    // [Hq, T], natural log
  const float* delta;  // [Hq, T]
  float* dq_acc;       // [T, Hq, D]
  bf16* dqkv;
  long ldd;
  int* err;
  // optional phase stamps (clock64) of CTA (0, 0, 0): [it < 64][event < 8]
  // of the softmax warp on TMEM lanes 0-31, [512 + it] the MMA issuer's
  // wait for P/dS; nullptr = off
  long long* dbg;
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// K-major 128-row operand of two 64-column swizzled boxes, k-step k (16 columns)
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int k) {
  return smem_desc_sw128(base + (k >> 2) * BOX + (k & 3) * 32, 16, 1024);
}
// MN-major operand: 128 rows of the K extent, 128 MN columns in two boxes
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int k) {
  return smem_desc_sw128(base + k * 2048, BOX, 1024);
}

__global__ void __launch_bounds__(192, 1)
    attn_bwd_pipe_kernel(const __grid_constant__ CUtensorMap tma_qkv,
                         const __grid_constant__ CUtensorMap tma_do,
                         const __grid_constant__ CUtensorMap tma_dq, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + TILE;
  uint8_t* sQ = sV + TILE;       // [2]
  uint8_t* sDO = sQ + 2 * TILE;
  uint8_t* sP = sDO + TILE;
  uint8_t* sDS = sP + TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDS + TILE);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;    // [2]
  uint64_t* q_free = bars + 3;    // [2]  dK of the buffer's last use completed
  uint64_t* do_full = bars + 5;
  uint64_t* do_free = bars + 6;   // dV of the current dO completed
  uint64_t* s_full = bars + 7;    // S and dP of the iteration computed
  uint64_t* pds_full = bars + 8;  // P and dS in shared memory (4 warps)
  uint64_t* dq_ready = bars + 9;  // dQ of the iteration in the dP columns
  uint64_t* dq_free = bars + 10;  // dQ drained (4 warps)
  uint64_t* mma_done = bars + 11; // every MMA of the CTA completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
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
  if (T1_OOB(tok0 + p.S - 1, p.T) || T1_OOB((long)(p.n_q + 2 * p.n_kv) * D - 1, p.ldd) ||
      T1_OOB(kb, nqb))
    return;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_free[i], 1);
    }
    mbar_init(do_full, 1);
    mbar_init(do_free, 1);
    mbar_init(s_full, 1);
    mbar_init(pds_full, 4);
    mbar_init(dq_ready, 1);
    mbar_init(dq_free, 4);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tma_qkv);
    prefetch_tensormap(&tma_do);
    prefetch_tensormap(&tma_dq);
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
        const int qrow = tok0 + (kb + it % per_head) * BM;
        const int qb = it & 1;
        if (it >= 2 && !mbar_wait(&q_free[qb], ((it >> 1) & 1) ^ 1)) {
          err.set(241);
          *abort_flag = 1;
          break;
        }
        uint8_t* q = sQ + qb * TILE;
        mbar_arrive_expect_tx(&q_full[qb], TILE);
        tma_load_2d(q, &tma_qkv, &q_full[qb], h * D, qrow);
        tma_load_2d(q + BOX, &tma_qkv, &q_full[qb], h * D + 64, qrow);
        if (it >= 1 && !mbar_wait(do_free, (it - 1) & 1)) {
          err.set(242);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(do_full, TILE);
        tma_load_2d(sDO, &tma_do, do_full, h * D, qrow);
        tma_load_2d(sDO + BOX, &tma_do, do_full, h * D + 64, qrow);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_KK = idesc_bf16_f32(BM, BN, false, false);  // S, dP
      constexpr uint32_t ID_MM = idesc_bf16_f32(BN, D, true, true);     // dV, dK
      constexpr uint32_t ID_KM = idesc_bf16_f32(BM, D, false, true);    // dQ
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), q0_addr = smem_u32(sQ);
      const uint32_t do_addr = smem_u32(sDO), p_addr = smem_u32(sP), ds_addr = smem_u32(sDS);
      // S(it) = Q K^T into the S columns, then dP(it) = dO V^T into the dP
      // columns once dO(it) arrived and dQ(it-1) left them
      auto issue_s_dp = [&](int it) -> bool {
        if (!mbar_wait(&q_full[it & 1], (it >> 1) & 1)) { err.set(243); return false; }
        tc_fence_after();
        const uint32_t q_addr = q0_addr + (it & 1) * TILE;
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          mma_bf16(t_s, kmajor_desc(q_addr, k), kmajor_desc(k_addr, k), ID_KK, k != 0);
        if (!mbar_wait(do_full, it & 1)) { err.set(244); return false; }
        if (it > 0 && !mbar_wait(dq_free, (it - 1) & 1)) { err.set(245); return false; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          mma_bf16(t_dp, kmajor_desc(do_addr, k), kmajor_desc(v_addr, k), ID_KK, k != 0);
        mma_commit(s_full);
        return true;
      };
      long long* dbg = (p.dbg != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) ? p.dbg
                                                                                                  : nullptr;
      bool ok = mbar_wait(kv_full, 0);
      if (!ok) err.set(246);
      if (ok && n_it > 0) ok = issue_s_dp(0);
      for (int it = 0; ok && it < n_it && !*abort_flag; ++it) {
        if (!mbar_wait(pds_full, it & 1)) { err.set(247); ok = false; break; }
        if (dbg != nullptr && it < 64) dbg[512 + it] = clock64();
        tc_fence_after();
        const uint32_t q_addr = q0_addr + (it & 1) * TILE;
        // dV += P^T dO: dO's buffer is free afterwards
#pragma unroll
        for (int k = 0; k < BM / 16; ++k)
          mma_bf16(t_dv, mnmajor_desc(p_addr, k), mnmajor_desc(do_addr, k), ID_MM, (it | k) != 0);
        mma_commit(do_free);
        // dQ = dS K into the dP columns (the softmax warps read dP already)
#pragma unroll
        for (int k = 0; k < BN / 16; ++k)
          mma_bf16(t_dp, kmajor_desc(ds_addr, k), mnmajor_desc(k_addr, k), ID_KM, k != 0);
        mma_commit(dq_ready);
        // dK += dS^T Q: this Q buffer is free afterwards
#pragma unroll
        for (int k = 0; k < BM / 16; ++k)
          mma_bf16(t_dk, mnmajor_desc(ds_addr, k), mnmajor_desc(q_addr, k), ID_MM, (it | k) != 0);
        mma_commit(&q_free[it & 1]);
        if (it + 1 < n_it && !issue_s_dp(it + 1)) { ok = false; break; }
      }
      mma_commit(mma_done);
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------------------------------- softmax / dQ drain / dK dV warps
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row of the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    long long* sdbg = (p.dbg != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 &&
                       quarter == 0 && lane == 0) ? p.dbg : nullptr;
    auto stamp = [&](int it, int e) {
      if (sdbg != nullptr && it < 64) sdbg[it * 8 + e] = clock64();
    };
    bool ok = true;
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
    // dQ of iteration `it` (in the dP columns) x scale -> dq_acc by TMA bulk
    // reduce-adds, staged through this warp's rows of the P buffer (free
    // here: dV(it) has read P, and the softmax writes P(it + 1) only after
    // the drain).  Per 64 columns two 32 x 32 fp32 boxes, 128B-swizzled: at
    // sP + 4 KB q and sP + 16 KB + 4 KB q, exactly the bytes of P rows
    // 32q .. 32q + 31 that this warp itself writes later.  One bulk reduce
    // per box instead of 32 vector atomics per thread.
    uint8_t* box_a = sP + quarter * 4096;
    uint8_t* box_b = sP + BOX + quarter * 4096;
    auto put_box = [&](uint8_t* box, const uint32_t (&u)[32]) {
      uint8_t* rowp = box + lane * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float4*>(rowp + ((j ^ (lane & 7)) << 4)) =
            make_float4(__uint_as_float(u[4 * j]) * p.scale, __uint_as_float(u[4 * j + 1]) * p.scale,
                        __uint_as_float(u[4 * j + 2]) * p.scale, __uint_as_float(u[4 * j + 3]) * p.scale);
    };
    auto drain_dq = [&](int it) {
      const int h = g * G + it / per_head;
      const int row0 = tok0 + (kb + it % per_head) * BM + quarter * 32;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t u0[32], u1[32];
        tmem_ld_32x32b_x32(t_dp + lane_base + hh * 64, u0);
        tmem_ld_32x32b_x32(t_dp + lane_base + hh * 64 + 32, u1);
        tmem_ld_wait();
        if (hh == 1) {
          // every dP column is read: the next dP may be computed
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(dq_free);
          // and the first half's reduces have read the boxes
          if (lane == 0) bulk_wait_group_read<0>();
          __syncwarp();
        }
        put_box(box_a, u0);
        put_box(box_b, u1);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&tma_dq, box_a, h * D + hh * 64, row0);
          tma_reduce_add_2d(&tma_dq, box_b, h * D + hh * 64 + 32, row0);
          bulk_commit_group();
        }
      }
      // the boxes are rows of P: the reduces must have read them
      if (lane == 0) bulk_wait_group_read<0>();
      __syncwarp();
    };
    for (int it = 0; it < n_it; ++it) {
      const int h = g * G + it / per_head;
      const int qpos = (kb + it % per_head) * BM + r;
      const bool q_ok = qpos < p.S;
      // issued before the drain below, so their latency hides behind it
      const float lse2 = q_ok ? p.lse[static_cast<long>(h) * p.T + tok0 + qpos] * LOG2E : 0.f;
      const float dlt = q_ok ? p.delta[static_cast<long>(h) * p.T + tok0 + qpos] : 0.f;
      stamp(it, 0);
      if (it > 0) {
        if (!wait_w(dq_ready, (it - 1) & 1, 248)) { ok = false; break; }
        stamp(it, 1);
        tc_fence_after();
        drain_dq(it - 1);
      }
      stamp(it, 2);
      if (!wait_w(s_full, it & 1, 249)) { ok = false; break; }
      stamp(it, 3);
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
      stamp(it, 4);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pds_full);
      stamp(it, 5);
    }
    if (ok && n_it > 0 && wait_w(dq_ready, (n_it - 1) & 1, 250)) {
      tc_fence_after();
      drain_dq(n_it - 1);
      if (wait_w(mma_done, 0, 251)) {
        tc_fence_after();
        // dK (scaled) and dV rows: TMEM lane r = key row r of the block
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

  if (warp >= 2 && lane == 0) bulk_wait_group_all();  // the dQ reduce-adds landed
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn_bwd2

T1_BOUNDS_READER(attention_bwd2)

// Phase-stamp buffer (int64 [>= 576] on the GPU) or undefined = off.
static torch::Tensor& attn_bwd2_debug() {
  static torch::Tensor t;
  return t;
}

void attn_bwd2_set_debug(torch::Tensor buf) {
  if (buf.defined() && buf.numel() > 0) {
    TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == torch::kInt64 && buf.is_contiguous() && buf.numel() >= 576,
                "phase-stamp buffer must be a contiguous CUDA int64 tensor of >= 576 elements");
    attn_bwd2_debug() = buf;
  } else {
    attn_bwd2_debug() = torch::Tensor();
  }
}

// Pipelined backward core: same contract as attention_bwd_tc_core.
void attention_bwd_pipe_core(torch::Tensor dout, torch::Tensor qkv, torch::Tensor lse,
                             torch::Tensor delta, torch::Tensor dq_acc, torch::Tensor dqkv, int64_t n_q,
                             int64_t n_kv, int64_t S) {
  const int64_t T = qkv.size(0), B = T / S;
  const CUtensorMap mq = make_map(qkv.data_ptr(), qkv.size(1), T, qkv.stride(0), 128);
  const CUtensorMap md = make_map(dout.data_ptr(), dout.size(1), T, dout.stride(0), 128);
  TORCH_CHECK(dq_acc.is_contiguous() && dq_acc.numel() == T * n_q * attn_bwd2::D, "dq_acc must be [T, Hq, D]");
  const CUtensorMap mdq = make_map_f32(dq_acc.data_ptr(), n_q * attn_bwd2::D, T, n_q * attn_bwd2::D);
  attn_bwd2::Params p;
  p.S = static_cast<int>(S);
  p.T = static_cast<int>(T);
  p.n_q = static_cast<int>(n_q);
  p.n_kv = static_cast<int>(n_kv);
  p.scale = 1.0f / std::sqrt(static_cast<float>(attn_bwd2::D));
  p.scale_log2 = p.scale * attn_bwd2::LOG2E;
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  p.ldd = dqkv.stride(0);
  p.err = gemm_error_word().data_ptr<int>();
  p.dbg = attn_bwd2_debug().defined() ? reinterpret_cast<long long*>(attn_bwd2_debug().data_ptr<int64_t>())
                                      : nullptr;
  static bool cfg = false;
  if (!cfg) {
    T1_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd2::attn_bwd_pipe_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, attn_bwd2::SMEM_BYTES));
    cfg = true;
  }
  dim3 grid((S + attn_bwd2::BN - 1) / attn_bwd2::BN, n_kv, B);
  attn_bwd2::attn_bwd_pipe_kernel<<<grid, 192, attn_bwd2::SMEM_BYTES, stream()>>>(mq, md, mdq, p);
  check_launch("attention_bwd_pipe");
  count_launch();
}

}  // namespace t1
