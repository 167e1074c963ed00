// Causal GQA attention forward on tcgen05, two query tiles per CTA in
// ping-pong (head_dim 128, fused qkv buffer [T, (Hq + 2 Hkv) * 128]).
// Same outputs as attn_fwd_tc_kernel (attention_tc.cu): o [T, Hq*128] bf16
// and lse [Hq, T] (natural log, 1/sqrt(d) included), so the backward
// kernels consume either.
//
// Why two tiles: with one 128-row tile per CTA the tensor core waits for the
// softmax of every key block (one softmax warp per scheduler, 128
// exponentials per thread per block).  Here a CTA owns 256 query rows as
// tiles A and B that share every K/V block; while the softmax warps of one
// tile work, the tensor core computes the other tile's S = Q K^T and P V.
//
// One CTA per (256-query block, head, sequence), heaviest blocks first;
// 320 threads:
//   warp 0      TMA producer: Q_A and Q_B once, then K_0, K_1, V_0, K_2,
//               V_1, ... through a 3-slot ring of 32 KB tiles (no multicast)
//   warp 1      TMEM owner (S_A | S_B | O_A | O_B, 512 columns) and the
//               single-thread MMA issuer, in the order
//                 S_A(0) S_B(0) { S_A(j+1) S_B(j+1) PV_A(j) PV_B(j) }
//               where S_t(j+1) starts as soon as tile t's softmax warps
//               have read S_t(j) into registers, so the next scores are
//               ready when a softmax finishes and the two tiles' softmax
//               phases overlap each other and the MMAs
//   warps 2-5   softmax of tile A, warps 6-9 softmax of tile B: thread =
//               query row = TMEM lane; scale, causal mask, running max/sum in
//               base 2 with lazy rescaling of O, P (bf16) into 128B-swizzled
//               shared memory for the P V MMA; final O / l and the LSE.
// Exponentials: on the MUFU unit (ex2.approx) by default; POLY (0-2) of
// every 8 can run on the FMA pipe instead as 2^x = 2^round(x) * p(x -
// round(x)), p a cubic interpolating 2^r at the four Chebyshev nodes of
// [-0.5, 0.5] (max relative error 1.0e-4, far below the bf16 rounding of P).
// Measured on B200 (B=4, S=1024 and B=2, S=4096): POLY 0 fastest, 1 within
// 2 %, 2 slower by 15-20 % (the extra registers spill).
// Every wait is bounded (sm100.cuh); a timeout writes the error word.
#include "common.cuh"
#include "sm100.cuh"

namespace t1 {

CUtensorMap make_map(const void* ptr, int64_t inner, int64_t outer, int64_t ld, int box_outer);
torch::Tensor& gemm_error_word();

namespace attn_tc2 {

using namespace sm100;
using bf16 = __nv_bfloat16;

constexpr int D = 128;
constexpr int BM = 128;            // query rows per tile (two tiles per CTA)
constexpr int BN = 128;            // keys per block
constexpr int BOX = 128 * 64 * 2;  // one 128-row x 64-column bf16 box: 16 KB
constexpr int TILE = 2 * BOX;      // 128 x 128 bf16: 32 KB
constexpr int RING = 3;            // K/V ring slots
constexpr int THREADS = 320;
constexpr float LOG2E = 1.4426950408889634f;
constexpr int SMEM_BYTES = 2 * TILE /*Q_A,Q_B*/ + RING * TILE /*K/V*/ + 2 * TILE /*P_A,P_B*/ + 1024 + 256;
static_assert(SMEM_BYTES <= 232448, "attention forward v2 exceeds 227 KB of shared memory");

struct Params {
  int S, T, n_q, n_kv;
  float scale_log2;  // log2(e) / sqrt(D)
  bf16* out;
  long ld_out;
  float* lse;
  int* err;
  // optional phase stamps (clock64) of the heaviest CTA of head 0,
  // sequence 0: [tile][block < 32][event < 8] for the softmax warp of each
  // tile whose lanes are TMEM quarter 2, then [512 + 2 * block + tile] for
  // the MMA issuer's P waits; nullptr = off
  long long* dbg;
};

__device__ __forceinline__ float ex2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA/ALU pipes.  x is clamped to >= -126 so the exponent add
// below stays in the normal/denormal range (smaller weights are below what
// a bf16 P can represent next to the row maximum anyway).  Round-to-nearest
// of x by the 1.5 * 2^23 addition trick: the low bits of t hold round(x), so
// (bits(t) << 23) is round(x) in the exponent field.
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -126.f);
  const float t = x + 12582912.f;
  const float r = x - (t - 12582912.f);  // [-0.5, 0.5]
  float p = fmaf(0.05583828315138817f, r, 0.2426394820213318f);
  p = fmaf(p, r, 0.6931367516517639f);
  p = fmaf(p, r, 0.9999245405197144f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int k) {
  return smem_desc_sw128(base + (k >> 2) * BOX + (k & 3) * 32, 16, 1024);
}

// warp-uniform bounded wait on an mbarrier phase; lane 0 polls
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          const ErrorSlot& err, int code) {
  int w = 0;
  if ((threadIdx.x & 31) == 0) {
    w = !*abort_flag && mbar_wait(bar, parity);
    if (!w && !*abort_flag) {
      err.set(code);
      *abort_flag = 1;
    }
  }
  return __shfl_sync(0xffffffffu, w, 0) != 0;
}

// Ring order: K_0, then K_{j+1}, V_j for j = 0, 1, ... (V_{n-1} last), so
// the next block's keys are resident before this block's values are done
// with: position of K_j is 0 (j = 0) or 2j - 1, of V_j 2j + 2 (or 2n - 1 for
// the last block).
__device__ __forceinline__ int pos_k(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int pos_v(int j, int n) { return j + 1 < n ? 2 * j + 2 : 2 * n - 1; }
__device__ __forceinline__ void ring_item(int i, int n, bool& is_v, int& blk) {
  if (i == 0) { is_v = false; blk = 0; return; }
  if (i == 2 * n - 1) { is_v = true; blk = n - 1; return; }
  is_v = (i & 1) == 0;          // even positions >= 2 hold V_{i/2 - 1}
  blk = is_v ? i / 2 - 1 : (i + 1) / 2;
}

template <int POLY>
__global__ void __launch_bounds__(THREADS, 1)
    attn_fwd_tc2_kernel(const __grid_constant__ CUtensorMap tma_qkv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                   // [2] tiles
  uint8_t* sR = sQ + 2 * TILE;          // [RING] K/V slots
  uint8_t* sP = sR + RING * TILE;       // [2] tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * TILE);
  uint64_t* q_full = bars + 0;
  uint64_t* r_full = bars + 1;   // [RING]
  uint64_t* r_empty = bars + 4;  // [RING]
  uint64_t* s_full = bars + 7;   // [2]  S_t(j) computed
  uint64_t* p_full = bars + 9;   // [2]  P_t(j) written (4 warps)
  uint64_t* p_empty = bars + 11; // [2]  P_t(j) V_j completed
  uint64_t* s_empty = bars + 13; // [2]  S_t(j) read into registers (4 warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const ErrorSlot err{p.err};
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const int qb2 = static_cast<int>(gridDim.z) - 1 - static_cast<int>(blockIdx.z);  // heavy first
  const int g = h / (p.n_q / p.n_kv);
  const int tok0 = b * p.S;
  const int q0 = qb2 * 2 * BM;
  const int nkb = (p.S + BN - 1) / BN;
  const int nB = min(2 * qb2 + 2, nkb);  // key blocks of tile B (rows q0+128..q0+255)
  const int nA = min(2 * qb2 + 1, nkb);  // key blocks of tile A
  if (T1_OOB(tok0 + p.S - 1, p.T) || T1_OOB((long)p.n_q * D - 1, p.ld_out)) return;
  long long* dbg = (p.dbg != nullptr && h == 0 && b == 0 && blockIdx.z == 0) ? p.dbg : nullptr;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < RING; ++s) {
      mbar_init(&r_full[s], 1);
      mbar_init(&r_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&p_empty[t], 1);
      mbar_init(&s_empty[t], 4);
    }
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
  const uint32_t t_s = tmem;        // S_A [0,128), S_B [128,256)
  const uint32_t t_o = tmem + 256;  // O_A [256,384), O_B [384,512)

  // ring item i: K_{i/2} (even i) or V_{i/2} (odd i); slot i % RING, its
  // (i / RING)-th use
  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (lane == 0) {
      const int qcol = h * D, kcol = (p.n_q + g) * D, vcol = (p.n_q + p.n_kv + g) * D;
      mbar_arrive_expect_tx(q_full, 2 * TILE);
      tma_load_2d(sQ, &tma_qkv, q_full, qcol, tok0 + q0);
      tma_load_2d(sQ + BOX, &tma_qkv, q_full, qcol + 64, tok0 + q0);
      tma_load_2d(sQ + TILE, &tma_qkv, q_full, qcol, tok0 + q0 + BM);
      tma_load_2d(sQ + TILE + BOX, &tma_qkv, q_full, qcol + 64, tok0 + q0 + BM);
      for (int i = 0; i < 2 * nB && !*abort_flag; ++i) {
        const int slot = i % RING;
        if (!mbar_wait(&r_empty[slot], ((i / RING) & 1) ^ 1)) {
          err.set(301);
          *abort_flag = 1;
          break;
        }
        uint8_t* dst = sR + slot * TILE;
        bool is_v;
        int blk;
        ring_item(i, nB, is_v, blk);
        const int col = is_v ? vcol : kcol;
        const int row = tok0 + blk * BN;
        mbar_arrive_expect_tx(&r_full[slot], TILE);
        tma_load_2d(dst, &tma_qkv, &r_full[slot], col, row);
        tma_load_2d(dst + BOX, &tma_qkv, &r_full[slot], col + 64, row);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BN, false, false);
      constexpr uint32_t IDESC_O = idesc_bf16_f32(BM, D, false, true);
      const uint32_t q_addr = smem_u32(sQ), r_addr = smem_u32(sR), p_addr = smem_u32(sP);
      int waited = -1;  // last ring item whose load was waited for
      auto item_ready = [&](int i) -> bool {
        for (; waited < i; ++waited) {
          const int it = waited + 1;
          if (!mbar_wait(&r_full[it % RING], (it / RING) & 1)) { err.set(302); return false; }
        }
        tc_fence_after();
        return true;
      };
      // S_t(j) = Q_t K_j^T
      auto issue_s = [&](int t, int j) {
        const uint32_t k_addr = r_addr + (pos_k(j) % RING) * TILE;
        const uint32_t qa = q_addr + t * TILE;
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          mma_bf16(t_s + t * BN, kmajor_desc(qa, k), kmajor_desc(k_addr, k), IDESC_S, k != 0);
        mma_commit(&s_full[t]);
      };
      // O_t += P_t(j) V_j, once the softmax warps of tile t published P_t(j)
      auto issue_pv = [&](int t, int j) -> bool {
        if (!mbar_wait(&p_full[t], j & 1)) { err.set(303 + t); return false; }
        if (dbg != nullptr && j < 32) dbg[512 + 2 * j + t] = clock64();
        tc_fence_after();
        const uint32_t v_addr = r_addr + (pos_v(j, nB) % RING) * TILE;
        const uint32_t pa = p_addr + t * TILE;
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          const uint64_t vd = smem_desc_sw128(v_addr + k * 2048, BOX, 1024);
          mma_bf16(t_o + t * D, kmajor_desc(pa, k), vd, IDESC_O, (j | k) != 0);
        }
        mma_commit(&p_empty[t]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0);
      if (!ok) err.set(305);
      if (ok) ok = item_ready(pos_k(0));
      if (ok) {
        issue_s(0, 0);
        issue_s(1, 0);
        mma_commit(&r_empty[pos_k(0) % RING]);  // K_0 read by both tiles
      }
      // per block j: the next scores of each tile as soon as its softmax
      // warps have read the current ones, then P V of both tiles
      for (int j = 0; ok && j < nB && !*abort_flag; ++j) {
        if (j + 1 < nB) {
          if (!item_ready(pos_k(j + 1))) { ok = false; break; }
          if (j + 1 < nA) {
            if (!mbar_wait(&s_empty[0], j & 1)) { err.set(312); ok = false; break; }
            tc_fence_after();
            issue_s(0, j + 1);
          }
          if (!mbar_wait(&s_empty[1], j & 1)) { err.set(313); ok = false; break; }
          tc_fence_after();
          issue_s(1, j + 1);
          mma_commit(&r_empty[pos_k(j + 1) % RING]);  // K_{j+1} read by both tiles
        }
        if (!item_ready(pos_v(j, nB))) { ok = false; break; }
        if (j < nA && !issue_pv(0, j)) { ok = false; break; }
        if (!issue_pv(1, j)) { ok = false; break; }
        mma_commit(&r_empty[pos_v(j, nB) % RING]);  // V_j read by both tiles
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------------ softmax warps
    const int t = (warp - 2) >> 2;            // tile: 0 = A (warps 2-5), 1 = B (6-9)
    const int quarter = warp & 3;             // TMEM lanes this warp may access
    const int r = quarter * 32 + lane;        // query row within the tile == TMEM lane
    const int qt0 = q0 + t * BM;              // first query position of the tile
    const int qpos = qt0 + r;
    const int n_t = t == 0 ? nA : nB;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_st = t_s + t * BN, t_ot = t_o + t * D;
    uint8_t* pbuf = sP + t * TILE;
    long long* st_dbg = (dbg != nullptr && warp == 2 + 4 * t && lane == 0) ? dbg + t * 256 : nullptr;
    auto stamp = [&](int j, int e) {
      if (st_dbg != nullptr && j < 32) st_dbg[j * 8 + e] = clock64();
    };
    float m = -INFINITY;  // running max (base 2, scale included)
    float l = 0.f;        // running sum
    bool ok = true;
    for (int j = 0; j < n_t; ++j) {
      stamp(j, 7);
      if (!warp_wait(&s_full[t], j & 1, abort_flag, err, 306 + t)) { ok = false; break; }
      stamp(j, 0);
      tc_fence_after();
      float sv[BN];
      {
        uint32_t u[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(t_st + lane_base + c * 32, u[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(u[c][i]);
      }
      // S_t is free for the next block's scores
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[t]);
      stamp(j, 1);
      // causal mask: only the tile's diagonal block (and a block crossing
      // the sequence end) needs it
      const int kbase = j * BN;
      if (kbase + BN - 1 > qt0 || kbase + BN > p.S) {
#pragma unroll
        for (int i = 0; i < BN; ++i) {
          const int kpos = kbase + i;
          if (kpos > qpos || kpos >= p.S) sv[i] = -INFINITY;
        }
      }
      float mxs[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mxs[k] = sv[k];
#pragma unroll
      for (int i = 8; i < BN; ++i) mxs[i & 7] = fmaxf(mxs[i & 7], sv[i]);
      float mx = fmaxf(fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3])),
                       fmaxf(fmaxf(mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7])));
      mx *= p.scale_log2;
      // lazy rescaling: the base m moves only when a row's block maximum
      // exceeds it by more than 8 (weights then stay below 2^8)
      float alpha = 1.f;
      if (__any_sync(0xffffffffu, mx > m + 8.f)) {
        const float m_new = fmaxf(m, mx);
        alpha = (m == -INFINITY) ? 0.f : ex2_mufu(m - m_new);
        m = m_new;
      }
      const float mb = (m == -INFINITY) ? 0.f : m;
      stamp(j, 2);
      float sums[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < BN; ++i) {
        const float x = fmaf(sv[i], p.scale_log2, -mb);
        const float e = ((i & 7) >= 8 - POLY) ? ex2_poly(x) : ex2_mufu(x);
        sv[i] = e;
        sums[i & 7] += e;
      }
      const float sum = ((sums[0] + sums[1]) + (sums[2] + sums[3])) + ((sums[4] + sums[5]) + (sums[6] + sums[7]));
      l = l * alpha + sum;
      stamp(j, 3);
      // P_t is single-buffered: P_t(j-1) V_{j-1} must have completed (it
      // has in practice: S_t(j) was issued after it), which also makes O_t
      // hold every block before j for the rescale below
      if (j > 0 && !warp_wait(&p_empty[t], (j - 1) & 1, abort_flag, err, 308 + t)) { ok = false; break; }
      stamp(j, 4);
#pragma unroll
      for (int c16 = 0; c16 < BN / 8; ++c16) {
        uint4 pk;
        __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
        for (int q = 0; q < 4; ++q) h2[q] = __floats2bfloat162_rn(sv[c16 * 8 + 2 * q], sv[c16 * 8 + 2 * q + 1]);
        const int box = c16 >> 3, u = c16 & 7;
        *reinterpret_cast<uint4*>(pbuf + box * BOX + r * 128 + ((u ^ (r & 7)) << 4)) = pk;
      }
      fence_proxy_async_smem();
      stamp(j, 5);
      tc_fence_after();
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        uint32_t u[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(t_ot + lane_base + c * 32, u[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int i = 0; i < 32; ++i) u[c][i] = __float_as_uint(__uint_as_float(u[c][i]) * alpha);
          tmem_st_32x32b_x32(t_ot + lane_base + c * 32, u[c]);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
      stamp(j, 6);
    }
    // epilogue: wait for the last P V, normalise, store O and the LSE
    if (ok && n_t > 0 && !warp_wait(&p_empty[t], (n_t - 1) & 1, abort_flag, err, 310 + t)) ok = false;
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool row_ok = qpos < p.S;
      bf16* orow = p.out + static_cast<long>(tok0 + qpos) * p.ld_out + h * D;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(t_ot + lane_base + c * 32, u);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 pk;
            __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              h2[q] = __floats2bfloat162_rn(__uint_as_float(u[v * 8 + 2 * q]) * inv,
                                            __uint_as_float(u[v * 8 + 2 * q + 1]) * inv);
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

}  // namespace attn_tc2

T1_BOUNDS_READER(attention_fwd2)

// Exponential split of the two-tile forward: how many of every 8 softmax
// exponentials run as the polynomial on the FMA pipe (0, 1 or 2); per
// process, T1_ATTN_POLY or attn_fwd2_set_poly().
static int& attn_poly() {
  static int v = [] {
    const char* e = std::getenv("T1_ATTN_POLY");
    return (e != nullptr && e[0] >= '0' && e[0] <= '2') ? e[0] - '0' : 0;
  }();
  return v;
}

void attn_fwd2_set_poly(int64_t n) {
  TORCH_CHECK(n >= 0 && n <= 2, "polynomial exponentials per 8: 0, 1 or 2");
  attn_poly() = static_cast<int>(n);
}

// Phase-stamp buffer (int64 [>= 576] on the GPU) or undefined = off.
static torch::Tensor& attn_fwd2_debug() {
  static torch::Tensor t;
  return t;
}

void attn_fwd2_set_debug(torch::Tensor buf) {
  if (buf.defined() && buf.numel() > 0) {
    TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == torch::kInt64 && buf.is_contiguous() && buf.numel() >= 576,
                "phase-stamp buffer must be a contiguous CUDA int64 tensor of >= 576 elements");
    attn_fwd2_debug() = buf;
  } else {
    attn_fwd2_debug() = torch::Tensor();
  }
}

template <int POLY>
static void launch_fwd2(const CUtensorMap& map, const attn_tc2::Params& p, dim3 grid) {
  static bool cfg = false;
  if (!cfg) {
    T1_CHECK_CUDA(cudaFuncSetAttribute(attn_tc2::attn_fwd_tc2_kernel<POLY>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, attn_tc2::SMEM_BYTES));
    cfg = true;
  }
  attn_tc2::attn_fwd_tc2_kernel<POLY><<<grid, attn_tc2::THREADS, attn_tc2::SMEM_BYTES, stream()>>>(map, p);
}

// Two-tile forward; the caller checked the qkv layout and that S is a
// multiple of 256.
std::vector<torch::Tensor> attention_fwd_tc2(torch::Tensor qkv, int64_t n_q, int64_t n_kv, int64_t S) {
  TORCH_CHECK(S % (2 * attn_tc2::BM) == 0, "two-tile attention forward needs seq_len % 256 == 0");
  const int64_t D = attn_tc2::D, T = qkv.size(0), B = T / S;
  auto out = torch::empty({T, n_q * D}, qkv.options());
  auto lse = torch::empty({n_q, T}, qkv.options().dtype(torch::kFloat32));
  const CUtensorMap map = make_map(qkv.data_ptr(), qkv.size(1), T, qkv.stride(0), 128);
  attn_tc2::Params p;
  p.S = static_cast<int>(S);
  p.T = static_cast<int>(T);
  p.n_q = static_cast<int>(n_q);
  p.n_kv = static_cast<int>(n_kv);
  p.scale_log2 = attn_tc2::LOG2E / std::sqrt(static_cast<float>(D));
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ld_out = out.stride(0);
  p.lse = lse.data_ptr<float>();
  p.err = gemm_error_word().data_ptr<int>();
  p.dbg = attn_fwd2_debug().defined() ? reinterpret_cast<long long*>(attn_fwd2_debug().data_ptr<int64_t>()) : nullptr;
  dim3 grid(n_q, B, S / (2 * attn_tc2::BM));
  switch (attn_poly()) {
    case 1: launch_fwd2<1>(map, p, grid); break;
    case 2: launch_fwd2<2>(map, p, grid); break;
    default: launch_fwd2<0>(map, p, grid); break;
  }
  check_launch("attention_fwd_tc2");
  count_launch();
  return {out, lse};
}

}  // namespace t1
