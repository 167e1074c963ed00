// tcgen05 GEMM kernel template (see gemm.cu for the design notes).  The
// AG=true instantiation adds two gather warps per CTA and per-tile waits on
// B-row arrival flags: the shard-mode all-gather fused with the QKV GEMM
// (fused_ag_gemm.cu).
#pragma once

#include "common.cuh"
#include "sm100.cuh"

namespace t1 {

using bf16 = __nv_bfloat16;
using namespace sm100;

namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 16;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;

enum Epilogue : int { kStore = 0, kAddResidual = 1 };

struct Params {
  int M, N, K;
  bf16* C;
  long ldc;
  const bf16* R;
  long ldr;
  int tiles_m, tiles_n, num_tiles, k_blocks;
  int* err;
  // RoPE fused into the epilogue (pair kernel, TMA stores, head_dim 128):
  // columns [0, rope_cols) are rotated by position (row % rope_S) with the
  // fp32 tables rope_cos / rope_sin [rope_S, 64]
  const float* rope_cos;
  const float* rope_sin;
  int rope_S, rope_cols;
  // Stream-K tail (pair kernel with the TMA-store epilogue): the tiles from
  // sk_tail0 on (the last, partial wave) are each split along K into two
  // pieces run by different clusters; the first writes its fp32 partial
  // accumulator to sk_ws and counts its arrival in sk_flags, the second
  // loads it, adds it before its epilogue and resets the counter.
  // sk_split == 1 (the default) leaves one work unit per tile.
  int sk_split = 1;
  int sk_tail0 = 0;
  int num_units = 0;         // sk_tail0 + (num_tiles - sk_tail0) * sk_split
  float* sk_ws = nullptr;    // [tail tile][cta 2][warp 4][slab 4][row 32][64] fp32
  int* sk_flags = nullptr;   // [tail tile][cta 2][quarter 4], zero between launches
};

// Work unit u of the pair kernel: its tile, k-block range [kb0, kb1) and
// stream-K piece (-1: the whole tile).
__device__ __forceinline__ void unit_info(const Params& p, int u, int& tile, int& kb0, int& kb1,
                                          int& piece) {
  if (p.sk_split <= 1 || u < p.sk_tail0) {
    tile = u;
    kb0 = 0;
    kb1 = p.k_blocks;
    piece = -1;
    return;
  }
  const int i = u - p.sk_tail0;
  tile = p.sk_tail0 + i / p.sk_split;
  piece = i % p.sk_split;
  kb0 = piece * p.k_blocks / p.sk_split;
  kb1 = (piece + 1) * p.k_blocks / p.sk_split;
}

// Fused all-gather (shard mode): extra parameters of the AG variant.
constexpr int kAgMaxRanks = 8;
constexpr int kAgMaxBlocks = 64;  // 256-row blocks of the gathered weight
struct AgParams {
  uint64_t peer[kAgMaxRanks];  // every rank's pool unit (the layer's flat bf16 buffer)
  uint64_t sig[kAgMaxRanks];   // every rank's signal pad for that buffer
  int rank, world;
  long shard_off, shard_n;     // this rank's shard of the layer (elements)
  const void* host_src;        // device view of the page-locked shard
  const void* host_src_lo;     // split master: the low plane
  int src_kind;                // 0 bf16 copy, 1 fp32 master, 2 split master (hi/lo planes)
  int skip_self;               // the source is this rank's own unit (placed there by the copy
                               // engine): store to the peers only
  uint32_t epoch;
  int n_blocks;                // 256-row blocks of B (= the QKV weight rows / 256)
  long block_elems;            // 256 * K
  uint8_t owners[kAgMaxBlocks];  // bitmask of ranks whose shard intersects block b
  int* counters;               // kAgMaxBlocks + 1 device ints, zero between launches
  uint64_t wait_ns;            // limit of every wait on a peer
};

__device__ __forceinline__ void raster(int tile, int tiles_m, int tiles_n, int& mb, int& nb) {
  const int group = GROUP_M * tiles_n;
  const int gid = tile / group;
  const int first_m = gid * GROUP_M;
  const int gsz = min(tiles_m - first_m, GROUP_M);
  const int in_group = tile % group;
  mb = first_m + in_group % gsz;
  nb = in_group / gsz;
}

// ---- signalling helpers of the AG variant (slots in the unit's signal pad:
// [0, W) free, [W, 2W) done, 2W + b*W + p: block b written by rank p)
__device__ __forceinline__ void ag_store_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ag_load_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool ag_wait_geq(const uint32_t* p, uint32_t epoch, uint64_t wait_ns) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t n = 0;
  while (ag_load_acquire(p) < epoch) {
    if ((++n & 255u) == 0 && globaltimer_ns() - t0 > wait_ns) return false;
  }
  return true;
}
__device__ __forceinline__ void ag_signal_all(const AgParams& ag, int slot) {
  for (int q = 0; q < ag.world; ++q)
    ag_store_release(reinterpret_cast<uint32_t*>(ag.sig[q]) + slot, ag.epoch);
}
__device__ __forceinline__ void ag_named_barrier() { asm volatile("bar.sync 1, 64;" ::: "memory"); }

// 8 elements of this rank's shard at `local` as bf16 (cast from the fp32
// master or rebuilt from split planes when the source is not bf16).
__device__ __forceinline__ int4 ag_load8(const AgParams& ag, long local) {
  int4 out;
  if (ag.src_kind == 0) {
    out = *reinterpret_cast<const int4*>(static_cast<const bf16*>(ag.host_src) + local);
  } else {
    float f[8];
    if (ag.src_kind == 1) {
      const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(ag.host_src) + local);
      float4 x = src[0], y = src[1];
      f[0] = x.x; f[1] = x.y; f[2] = x.z; f[3] = x.w;
      f[4] = y.x; f[5] = y.y; f[6] = y.z; f[7] = y.w;
    } else {
      int4 hv = *reinterpret_cast<const int4*>(static_cast<const uint16_t*>(ag.host_src) + local);
      int4 lv = *reinterpret_cast<const int4*>(static_cast<const uint16_t*>(ag.host_src_lo) + local);
      const uint16_t* h = reinterpret_cast<const uint16_t*>(&hv);
      const uint16_t* l = reinterpret_cast<const uint16_t*>(&lv);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        f[k] = __uint_as_float(((static_cast<uint32_t>(h[k]) << 16) | l[k]) - 0x8000u);
    }
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
  }
  return out;
}

// Copy elements [b, e) of the layer (inside this rank's shard) to every peer,
// 8 elements per vector, 64 gather threads per CTA, 4 vectors per thread in
// flight (loads issued together ahead of the peer stores).
__device__ __forceinline__ void ag_copy(const AgParams& ag, long b, long e, int gt) {
  const long v0 = b >> 3, v1 = e >> 3;
  constexpr int kU = 4;
  for (long vb = v0 + gt; vb < v1; vb += 64 * kU) {
    int4 out[kU];
    bool ok[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long v = vb + 64 * u;
      const long local = 8 * v - ag.shard_off;
      ok[u] = v < v1 && !T1_OOB(local, ag.shard_n) && !T1_OOB(local + 7, ag.shard_n);
      if (ok[u]) out[u] = ag_load8(ag, local);
    }
    for (int q = 0; q < ag.world; ++q) {
      if (ag.skip_self && q == ag.rank) continue;
#pragma unroll
      for (int u = 0; u < kU; ++u)
        if (ok[u]) *reinterpret_cast<int4*>(reinterpret_cast<bf16*>(ag.peer[q]) + 8 * (vb + 64 * u)) = out[u];
    }
  }
}

// This CTA's share of [b, e): an even split over gridDim.x CTAs (8-aligned).
__device__ __forceinline__ void ag_cta_range(long b, long e, long& cb, long& ce) {
  const long nv = (e - b) >> 3;
  const long per = (nv + gridDim.x - 1) / gridDim.x;
  cb = b + 8 * min(nv, per * static_cast<long>(blockIdx.x));
  ce = b + 8 * min(nv, per * static_cast<long>(blockIdx.x + 1));
}

// Gather warps (threads 192-255) of the AG variants: copy this rank's
// shard of the layer from host memory into every peer's unit, one 256-row
// block of the QKV weight after another, publishing each block's arrival
// in every peer's signal pad, then everything after the QKV rows; the last
// CTA waits until every peer's shard has landed here.
__device__ __forceinline__ void ag_gather_warps(const AgParams& ag, const ErrorSlot& err,
                                                volatile int* abort_flag) {
    // ------------------------------------------- gather warps (AG only)
    const int gt = threadIdx.x - 192;
    const uint32_t* pad = reinterpret_cast<const uint32_t*>(ag.sig[ag.rank]);
    if (blockIdx.x == 0 && gt == 0) ag_signal_all(ag, ag.rank);  // my unit is free
    __shared__ int ag_ok;
    if (gt == 0) {
      bool ok = true;
      for (int q = 0; q < ag.world && ok; ++q) ok = ag_wait_geq(pad + q, ag.epoch, ag.wait_ns);
      ag_ok = ok;
      if (!ok) {
        err.set(122);
        *abort_flag = 1;
      }
    }
    ag_named_barrier();
    if (ag_ok) {
      const long s0 = ag.shard_off, s1 = ag.shard_off + ag.shard_n;
      for (int b = 0; b <= ag.n_blocks; ++b) {
        // block b of the weight rows, then (b == n_blocks) everything after them
        const long lo = max(s0, static_cast<long>(b) * ag.block_elems);
        const long hi = b < ag.n_blocks ? min(s1, static_cast<long>(b + 1) * ag.block_elems) : s1;
        if (lo >= hi) continue;
        long cb, ce;
        ag_cta_range(lo, hi, cb, ce);
        ag_copy(ag, cb, ce, gt);
        if (b < ag.n_blocks) {
          __threadfence_system();
          ag_named_barrier();
          if (gt == 0) {
            if (atomicAdd(&ag.counters[b], 1) == static_cast<int>(gridDim.x) - 1) {
              atomicExch(&ag.counters[b], 0);
              ag_signal_all(ag, 2 * ag.world + b * ag.world + ag.rank);
            }
          }
        }
      }
      // tail elements (shard_n % 8) by CTA 0
      if (blockIdx.x == 0) {
        for (long j = ((s1 >> 3) << 3) + gt; j < s1; j += 64) {
          const long local = j - s0;
          bf16 v;
          if (ag.src_kind == 0) {
            v = static_cast<const bf16*>(ag.host_src)[local];
          } else if (ag.src_kind == 1) {
            v = __float2bfloat16_rn(static_cast<const float*>(ag.host_src)[local]);
          } else {
            const uint32_t b = ((static_cast<uint32_t>(static_cast<const uint16_t*>(ag.host_src)[local]) << 16) |
                                static_cast<const uint16_t*>(ag.host_src_lo)[local]) - 0x8000u;
            v = __float2bfloat16_rn(__uint_as_float(b));
          }
          for (int q = 0; q < ag.world; ++q)
            if (!(ag.skip_self && q == ag.rank)) reinterpret_cast<bf16*>(ag.peer[q])[j] = v;
        }
      }
      __threadfence_system();
      ag_named_barrier();
      if (gt == 0 && atomicAdd(&ag.counters[kAgMaxBlocks], 1) == static_cast<int>(gridDim.x) - 1) {
        // last CTA: everything this rank owns is out; wait for every peer's
        ag_signal_all(ag, ag.world + ag.rank);
        bool ok = true;
        for (int q = 0; q < ag.world && ok; ++q) ok = ag_wait_geq(pad + ag.world + q, ag.epoch, ag.wait_ns);
        if (!ok) err.set(123);
        atomicExch(&ag.counters[kAgMaxBlocks], 0);
      }
    }
}

template <bool A_MN, bool B_MN, int EPI, bool AG>
__global__ void __launch_bounds__(AG ? 256 : 192, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tma_a,
                     const __grid_constant__ CUtensorMap tma_b, const Params p, const AgParams ag) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const ErrorSlot err{p.err};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);  // one arrival per epilogue warp
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tma_a);
    prefetch_tensormap(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed_parity[STAGES];
      bool armed[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) armed[s] = false;
      for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
        int mb, nb;
        raster(tile, p.tiles_m, p.tiles_n, mb, nb);
        if (AG && nb < ag.n_blocks) {
          // the B rows of this tile must have arrived from their owner ranks
          const uint32_t* pad = reinterpret_cast<const uint32_t*>(ag.sig[ag.rank]);
          bool ok = true;
          for (int q = 0; q < ag.world && ok; ++q)
            if (ag.owners[nb] & (1u << q))
              ok = ag_wait_geq(pad + 2 * ag.world + nb * ag.world + q, ag.epoch, ag.wait_ns);
          if (!ok) {
            err.set(121);
            *abort_flag = 1;
            break;
          }
          asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) {
            err.set(101);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          armed[stage] = true;
          armed_parity[stage] = phase;
          uint8_t* a = sA + stage * A_BYTES;
          uint8_t* b = sB + stage * B_BYTES;
          const int k0 = kb * BK;
          if (!A_MN) {
            tma_load_2d(a, &tma_a, &full[stage], k0, mb * BM);
          } else {
            tma_load_2d(a, &tma_a, &full[stage], mb * BM, k0);
            tma_load_2d(a + 8192, &tma_a, &full[stage], mb * BM + 64, k0);
          }
          if (!B_MN) {
            tma_load_2d(b, &tma_b, &full[stage], k0, nb * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(b + j * 8192, &tma_b, &full[stage], nb * BN + 64 * j, k0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // On abort, let every load this thread issued land before the CTA
      // exits (each wait is itself bounded).
      if (*abort_flag) {
        for (int s = 0; s < STAGES; ++s)
          if (armed[s]) mbar_wait(&full[s], armed_parity[s]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) {
          err.set(102);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase)) {
            err.set(103);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? smem_desc_sw128(a_addr + k * 2048, 8192, 1024)
                                     : smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc_sw128(b_addr + k * 2048, 8192, 1024)
                                     : smem_desc_sw128(b_addr + k * 32, 16, 1024);
            mma_bf16(d_tmem, ad, bd, IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
      }
    }
  } else if (AG && warp >= 6) {
    ag_gather_warps(ag, err, abort_flag);
  } else {
    // --------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int local = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      // one lane waits and the warp follows it, so the warp never diverges
      // around the .sync.aligned TMEM loads below
      int ok = 0;
      if (lane == 0) {
        ok = !*abort_flag;
        if (ok && !mbar_wait(&tfull[acc], acc_phase)) {
          err.set(104);
          *abort_flag = 1;
          ok = 0;
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      tc_fence_after();
      int mb, nb;
      raster(tile, p.tiles_m, p.tiles_n, mb, nb);
      const int row = mb * BM + q * 32 + lane;
      const bool row_ok = row < p.M;
      bf16* crow = p.C + static_cast<long>(row) * p.ldc;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN + c, r);
        tmem_ld_wait();
        const int col0 = nb * BN + c;
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
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm

}  // namespace t1
