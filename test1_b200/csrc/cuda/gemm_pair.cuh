// tcgen05 GEMM on CTA pairs (cta_group::2): the pair computes a 256 x 256
// tile with one MMA stream issued by the even ("leader") CTA.  Each CTA
// stages only its own half of the tile's operands (128 rows of A and 128
// rows of B per k-block: 32 KB instead of the 48 KB a single CTA needs for
// 128 x 256), so shared-memory fill traffic from L2 per FLOP drops by a
// third -- the single-CTA kernel (gemm_core.cuh) is bound by exactly that
// traffic.  Accumulators: 256 x 256 fp32 split over both CTAs' TMEM (each
// holds its 128 rows), double-buffered (2 x 256 columns).
//
// Pair protocol (all waits bounded, see sm100.cuh):
//   full[s]    leader's barrier; the leader arms it with both CTAs' bytes,
//              both CTAs' TMA loads count on it (.cta_group::2 form)
//   empty[s]   per CTA; the leader's MMA commit arrives on both (mask 0b11)
//   tfull[a]   per CTA; accumulator a finished (commit to both)
//   tempty[a]  leader's; the 4 epilogue warps of each CTA arrive (count 8)
// No TMA load uses multicast.
//
// Epilogue forms:
//   register stores (TMA_EPI = false): each thread rounds its row of the
//     accumulator and stores it with 16-byte global stores (32 rows per warp
//     instruction);
//   TMA stores (TMA_EPI = true): each epilogue warp owns two 4 KB shared
//     buffers of 32 rows x 64 columns in the 128B-swizzled layout; per
//     64-column slab it reads the accumulator from TMEM, adds the residual
//     (TMA-loaded into the same buffer), rounds to bf16 into the buffer and
//     issues one bulk tensor store, double-buffered against the next slab.
//     The accumulator is handed back to the MMA warp as soon as its last
//     TMEM load finished, before the stores complete.
//   ROPE (with TMA stores): the QKV projection's epilogue rotates the q and
//     k heads (head_dim 128, rotate-half pairs (j, j + 64), angle of row
//     position % S) on the fp32 accumulator before the one bf16 rounding;
//     it works a whole head (two slabs) at a time.
#pragma once

#include "gemm_core.cuh"

namespace t1 {
namespace gemm {

constexpr int PAIR_BM = 256;
constexpr int PAIR_BN = 256;
constexpr int PAIR_HALF = 128;
constexpr int PAIR_STAGES = 6;
constexpr int PAIR_A_BYTES = PAIR_HALF * BK * 2;
constexpr int PAIR_B_BYTES = PAIR_HALF * BK * 2;
constexpr int PAIR_STAGE_BYTES = PAIR_A_BYTES + PAIR_B_BYTES;
constexpr int PAIR_SMEM_BYTES = PAIR_STAGES * PAIR_STAGE_BYTES + 1024 + 256;
constexpr int PAIR_EPI_BUF = 32 * 64 * 2;                      // one 32 x 64 bf16 slab: 4 KB
constexpr int PAIR_EPI_BYTES = 4 /*warps*/ * 2 * PAIR_EPI_BUF;  // 32 KB
constexpr int PAIR_SMEM_BYTES_TMA = PAIR_SMEM_BYTES + PAIR_EPI_BYTES;
static_assert(PAIR_SMEM_BYTES_TMA <= 232448, "pair GEMM with TMA epilogue exceeds 227 KB of shared memory");

// ---- stream-K tail helpers (see Params::sk_split)
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until *flag reaches target (false after the wait limit).
__device__ __forceinline__ bool sk_wait(const int* flag, int target) {
  if (ld_acquire_gpu(flag) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t n = 0;
  while (ld_acquire_gpu(flag) < target) {
    __nanosleep(128);
    if ((++n & 255u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

// Adds the first piece's partial sums of accumulator columns [c, c + 32)
// of row `lane` from the staged [slab][row][64] block (swizzled as written).
__device__ __forceinline__ void sk_add32(uint32_t (&r)[32], const uint8_t* stage, int c, int lane) {
  const float4* row = reinterpret_cast<const float4*>(stage + (c >> 6) * 8192 + lane * 256);
  const int half = (c >> 5) & 1;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 v = row[(half * 8 + j) ^ (lane & 7)];
    r[4 * j + 0] = __float_as_uint(__uint_as_float(r[4 * j + 0]) + v.x);
    r[4 * j + 1] = __float_as_uint(__uint_as_float(r[4 * j + 1]) + v.y);
    r[4 * j + 2] = __float_as_uint(__uint_as_float(r[4 * j + 2]) + v.z);
    r[4 * j + 3] = __float_as_uint(__uint_as_float(r[4 * j + 3]) + v.w);
  }
}

constexpr size_t kSkPartFloats = 2 * PAIR_HALF * PAIR_BN;  // one split tile's partial (both CTAs)

// AG = true: the shard-mode fused all-gather variant (see gemm_core.cuh and
// fused_ag_gemm.cu): two more warps per CTA copy this rank's host shard of
// the layer into every peer's unit, and the producers wait for the B rows
// of a tile to arrive before loading them.
template <bool A_MN, bool B_MN, int EPI, bool AG = false, bool TMA_EPI = false, bool ROPE = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(AG ? 256 : 192, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a,
                     const __grid_constant__ CUtensorMap tma_b, const Params p, const AgParams ag,
                     const __grid_constant__ CUtensorMap tma_c, const __grid_constant__ CUtensorMap tma_r) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + PAIR_STAGES * PAIR_A_BYTES;
  uint8_t* sE = sB + PAIR_STAGES * PAIR_B_BYTES;  // epilogue buffers (TMA_EPI), 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(sE + (TMA_EPI ? PAIR_EPI_BYTES : 0));
  uint64_t* empty = full + PAIR_STAGES;
  uint64_t* tfull = empty + PAIR_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* rbar = tempty + 2;  // [4] residual loads of the TMA epilogue, one per warp
  uint64_t* skbar = rbar + 4;   // [4] stream-K partial loads, one per warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(skbar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();  // 0 = leader
  const int cluster = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;
  const ErrorSlot err{p.err};

  if (threadIdx.x == 0) {
    for (int s = 0; s < PAIR_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // 4 epilogue warps x 2 CTAs
    }
    for (int w = 0; w < 4; ++w) {
      mbar_init(&rbar[w], 1);
      mbar_init(&skbar[w], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tma_a);
    prefetch_tensormap(&tma_b);
    if (TMA_EPI) {
      prefetch_tensormap(&tma_c);
      if (EPI == kAddResidual) prefetch_tensormap(&tma_r);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_units = p.sk_split > 1 ? p.num_units : p.num_tiles;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int u = cluster; u < num_units && !*abort_flag; u += nclusters) {
        int tile, kb0, kb1, piece;
        unit_info(p, u, tile, kb0, kb1, piece);
        int mb, nb;
        raster(tile, p.tiles_m, p.tiles_n, mb, nb);
        const int row_a = mb * PAIR_BM + static_cast<int>(crank) * PAIR_HALF;
        const int row_b = nb * PAIR_BN + static_cast<int>(crank) * PAIR_HALF;
        if (AG && nb < ag.n_blocks) {
          // the B rows of this tile must have arrived from their owner ranks
          const uint32_t* pad = reinterpret_cast<const uint32_t*>(ag.sig[ag.rank]);
          bool ok = true;
          for (int q = 0; q < ag.world && ok; ++q)
            if (ag.owners[nb] & (1u << q))
              ok = ag_wait_geq(pad + 2 * ag.world + nb * ag.world + q, ag.epoch, ag.wait_ns);
          if (!ok) {
            err.set(115);
            *abort_flag = 1;
            break;
          }
          asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) {
            err.set(111);
            *abort_flag = 1;
            break;
          }
          const uint32_t lfull = mapa_shared(smem_u32(&full[stage]), 0);
          if (crank == 0) mbar_arrive_expect_tx(&full[stage], 2 * PAIR_STAGE_BYTES);
          uint8_t* a = sA + stage * PAIR_A_BYTES;
          uint8_t* b = sB + stage * PAIR_B_BYTES;
          const int k0 = kb * BK;
          if (!A_MN) {
            tma_load_2d_pair(a, &tma_a, lfull, k0, row_a);
          } else {
            tma_load_2d_pair(a, &tma_a, lfull, row_a, k0);
            tma_load_2d_pair(a + 8192, &tma_a, lfull, row_a + 64, k0);
          }
          if (!B_MN) {
            tma_load_2d_pair(b, &tma_b, lfull, k0, row_b);
          } else {
            tma_load_2d_pair(b, &tma_b, lfull, row_b, k0);
            tma_load_2d_pair(b + 8192, &tma_b, lfull, row_b + 64, k0);
          }
          if (++stage == PAIR_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------- MMA issuer (leader only)
    if (lane == 0 && crank == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(PAIR_BM, PAIR_BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int u = cluster; u < num_units && !*abort_flag; u += nclusters, ++local) {
        int tile, kb0, kb1, piece;
        unit_info(p, u, tile, kb0, kb1, piece);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) {
          err.set(112);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * PAIR_BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase)) {
            err.set(113);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * PAIR_A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * PAIR_B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? smem_desc_sw128(a_addr + k * 2048, 8192, 1024)
                                     : smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc_sw128(b_addr + k * 2048, 8192, 1024)
                                     : smem_desc_sw128(b_addr + k * 32, 16, 1024);
            mma_bf16_pair(d_tmem, ad, bd, IDESC, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          mma_commit_pair(&empty[stage], 0x3);
          if (++stage == PAIR_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair(&tfull[acc], 0x3);
      }
    }
  } else if (AG && warp >= 6) {
    ag_gather_warps(ag, err, abort_flag);
  } else if (TMA_EPI) {
    // ------------------------------------------- epilogue (TMA stores)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint8_t* wbuf = sE + q * 2 * PAIR_EPI_BUF;
    const uint32_t leader_tempty0 = mapa_shared(smem_u32(&tempty[0]), 0);
    const uint32_t leader_tempty1 = mapa_shared(smem_u32(&tempty[1]), 0);
    uint32_t rphase = 0;
    int bi = 0;
    int local = 0;
    for (int u = cluster; u < num_units; u += nclusters, ++local) {
      int tile, kb0, kb1, piece;
      unit_info(p, u, tile, kb0, kb1, piece);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      int ok = 0;
      if (lane == 0) {
        ok = !*abort_flag;
        if (ok && !mbar_wait(&tfull[acc], acc_phase)) {
          err.set(114);
          *abort_flag = 1;
          ok = 0;
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      tc_fence_after();
      int mb, nb;
      raster(tile, p.tiles_m, p.tiles_n, mb, nb);
      const int row0 = mb * PAIR_BM + static_cast<int>(crank) * PAIR_HALF + q * 32;
      bool failed = false;
      // stream-K (split in two): the first piece writes its partial sums and
      // is done; the last piece brings them into shared memory with one bulk
      // copy per warp and adds them on the way (sk_stage != nullptr)
      const bool sk_writer = piece == 0;
      const uint8_t* sk_stage = nullptr;
      if (piece >= 0) {
        const int ti = tile - p.sk_tail0;
        // this warp's 32 rows of the partial: [slab 4][row 32][64 floats], the
        // 16-byte units of a row XOR-swizzled by the row (lane & 7)
        float* wsw = p.sk_ws + (static_cast<size_t>(ti) * 2 + crank) * kSkPartFloats / 2 +
                     static_cast<size_t>(q) * (32 * PAIR_BN);
        int* flag = p.sk_flags + (ti * 2 + static_cast<int>(crank)) * 4 + q;
        if (sk_writer) {
#pragma unroll 1
          for (int c = 0; c < PAIR_BN; c += 32) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * PAIR_BN + c, r);
            tmem_ld_wait();
            if (c + 32 == PAIR_BN) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_cluster(acc ? leader_tempty1 : leader_tempty0);
            }
            float4* row = reinterpret_cast<float4*>(wsw + (c >> 6) * 2048 + lane * 64);
            const int half = (c >> 5) & 1;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              __stcg(row + ((half * 8 + j) ^ (lane & 7)),
                     make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                 __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
          }
          __threadfence();
          __syncwarp();
          if (lane == 0) red_release_gpu_add(flag, 1);
          continue;
        }
        // the last piece is this cluster's last unit: the operand ring is
        // idle (every MMA that read it completed), 32 KB of it per warp
        uint8_t* stage_buf = sA + q * (32 * PAIR_BN * 4);
        int okf = 0;
        if (lane == 0) {
          okf = sk_wait(flag, 1);
          if (okf) {
            *flag = 0;  // consumed; the next launch starts from zero
            asm volatile("fence.proxy.async.global;" ::: "memory");
            mbar_arrive_expect_tx(&skbar[q], 32 * PAIR_BN * 4);
            bulk_load_1d(stage_buf, wsw, 32 * PAIR_BN * 4, &skbar[q]);
            okf = mbar_wait(&skbar[q], 0);
          }
          if (!okf) {
            err.set(117);
            *abort_flag = 1;
          }
        }
        if (!__shfl_sync(0xffffffffu, okf, 0)) break;
        sk_stage = stage_buf;
      }
      if (ROPE) {
        // one head (128 columns, two slabs) per step; both buffers are
        // rewritten, so every earlier store must have read them
#pragma unroll 1
        for (int c = 0; c < PAIR_BN; c += 128) {
          const int col0 = nb * PAIR_BN + c;
          const bool live = col0 < p.N && row0 < p.M;
          if (lane == 0) bulk_wait_group_read<0>();
          __syncwarp();
          uint32_t r[4][32];
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * PAIR_BN + c;
#pragma unroll
          for (int k = 0; k < 4; ++k) tmem_ld_32x32b_x32(taddr + 32 * k, r[k]);
          tmem_ld_wait();
          if (sk_stage != nullptr) {
#pragma unroll
            for (int k = 0; k < 4; ++k) sk_add32(r[k], sk_stage, c + 32 * k, lane);
          }
          if (c + 128 == PAIR_BN) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc ? leader_tempty1 : leader_tempty0);
          }
          if (!live) continue;
          if (col0 < p.rope_cols) {
            const int row = min(row0 + lane, p.M - 1);
            const int pos = row % p.rope_S;
            const float4* cp = reinterpret_cast<const float4*>(p.rope_cos + static_cast<size_t>(pos) * 64);
            const float4* sp = reinterpret_cast<const float4*>(p.rope_sin + static_cast<size_t>(pos) * 64);
#pragma unroll
            for (int j4 = 0; j4 < 16; ++j4) {
              const float4 cv = __ldg(cp + j4), sv = __ldg(sp + j4);
              const float cc[4] = {cv.x, cv.y, cv.z, cv.w};
              const float ss[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int j = 4 * j4 + u;
                const float x1 = __uint_as_float(r[j >> 5][j & 31]);
                const float x2 = __uint_as_float(r[(j + 64) >> 5][(j + 64) & 31]);
                r[j >> 5][j & 31] = __float_as_uint(x1 * cc[u] - x2 * ss[u]);
                r[(j + 64) >> 5][(j + 64) & 31] = __float_as_uint(x2 * cc[u] + x1 * ss[u]);
              }
            }
          }
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint8_t* buf = wbuf + hh * PAIR_EPI_BUF;
            uint8_t* rowp = buf + lane * 128;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              uint4 ov;
              __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
              for (int k = 0; k < 4; ++k)
                oh[k] = __floats2bfloat162_rn(__uint_as_float(r[2 * hh + (j >> 2)][(j & 3) * 8 + 2 * k]),
                                              __uint_as_float(r[2 * hh + (j >> 2)][(j & 3) * 8 + 2 * k + 1]));
              *reinterpret_cast<uint4*>(rowp + ((j ^ (lane & 7)) << 4)) = ov;
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tma_c, wbuf, col0, row0);
            if (col0 + 64 < p.N) tma_store_2d(&tma_c, wbuf + PAIR_EPI_BUF, col0 + 64, row0);
            bulk_commit_group();
          }
        }
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < PAIR_BN; c += 64) {
        uint8_t* buf = wbuf + bi * PAIR_EPI_BUF;
        const int col0 = nb * PAIR_BN + c;
        const bool live = col0 < p.N && row0 < p.M;  // a slab wholly outside C is skipped
        // the store issued from this buffer two slabs ago has read it
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        if (EPI == kAddResidual && live && lane == 0) {
          mbar_arrive_expect_tx(&rbar[q], PAIR_EPI_BUF);
          tma_load_2d(buf, &tma_r, &rbar[q], col0, row0);
        }
        uint32_t r0[32], r1[32];
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * PAIR_BN + c;
        tmem_ld_32x32b_x32(taddr, r0);
        tmem_ld_32x32b_x32(taddr + 32, r1);
        tmem_ld_wait();
        if (sk_stage != nullptr) {
          sk_add32(r0, sk_stage, c, lane);
          sk_add32(r1, sk_stage, c + 32, lane);
        }
        if (c + 64 == PAIR_BN) {
          // every TMEM read of this accumulator is done: hand it back now
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acc ? leader_tempty1 : leader_tempty0);
        }
        if (EPI == kAddResidual && live) {
          int okr = 0;
          if (lane == 0) okr = mbar_wait(&rbar[q], rphase);
          rphase ^= 1;
          if (!__shfl_sync(0xffffffffu, okr, 0)) {
            if (lane == 0) {
              err.set(116);
              *abort_flag = 1;
            }
            failed = true;
            break;
          }
        }
        if (live) {
          uint8_t* rowp = buf + lane * 128;  // row `lane` of the slab
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4* slot = reinterpret_cast<uint4*>(rowp + ((j ^ (lane & 7)) << 4));
            float f[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) f[k] = __uint_as_float(j < 4 ? r0[8 * j + k] : r1[8 * (j - 4) + k]);
            if (EPI == kAddResidual) {
              uint4 rv = *slot;
              const __nv_bfloat162* rh = reinterpret_cast<const __nv_bfloat162*>(&rv);
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float2 t = __bfloat1622float2(rh[k]);
                f[2 * k] += t.x;
                f[2 * k + 1] += t.y;
              }
            }
            uint4 ov;
            __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
            for (int k = 0; k < 4; ++k) oh[k] = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
            *slot = ov;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tma_c, buf, col0, row0);
            bulk_commit_group();
          }
          bi ^= 1;
        }
      }
      if (failed) break;
    }
    // every store of this warp completed before the CTA may exit
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
  } else {
    // --------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t leader_tempty0 = mapa_shared(smem_u32(&tempty[0]), 0);
    const uint32_t leader_tempty1 = mapa_shared(smem_u32(&tempty[1]), 0);
    int local = 0;
    for (int tile = cluster; tile < num_units; tile += nclusters, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      // one lane waits and the warp follows it, so the warp never diverges
      // around the .sync.aligned TMEM loads below
      int ok = 0;
      if (lane == 0) {
        ok = !*abort_flag;
        if (ok && !mbar_wait(&tfull[acc], acc_phase)) {
          err.set(114);
          *abort_flag = 1;
          ok = 0;
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      tc_fence_after();
      int mb, nb;
      raster(tile, p.tiles_m, p.tiles_n, mb, nb);
      const int row = mb * PAIR_BM + static_cast<int>(crank) * PAIR_HALF + q * 32 + lane;
      const bool row_ok = row < p.M;
      bf16* crow = p.C + static_cast<long>(row) * p.ldc;
#pragma unroll 1
      for (int c = 0; c < PAIR_BN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * PAIR_BN + c, r);
        tmem_ld_wait();
        const int col0 = nb * PAIR_BN + c;
        if (row_ok) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const int col = col0 + 8 * v;
            if (col < p.N && !T1_OOB(col + 7, p.ldc)) {
              float f[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(r[8 * v + j]);
              if (EPI == kAddResidual) {
                float rv[8];
                load8(p.R + static_cast<long>(row) * p.ldr + col, rv);
#pragma unroll
                for (int j = 0; j < 8; ++j) f[j] += rv[j];
              }
              store8(crow + col, f);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? leader_tempty1 : leader_tempty0);
    }
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync();  // neither CTA leaves while the pair still uses its smem / TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm
}  // namespace t1
