// Causal grouped-query attention, forward and backward, head_dim 128, on
// the fused qkv buffer [T, (Hq + 2 Hkv) * 128] (T = batch * S tokens).
//
// FlashAttention-2 dataflow with warp-level bf16 tensor-core MMAs
// (mma.sync m16n8k16, fp32 accumulation): 64-row query tiles x 64-key tiles,
// online softmax in base 2, P kept in registers as the A operand of P*V,
// K/V (and Q/dO in the backward) double-buffered in XOR-swizzled shared
// memory through cp.async.  The backward walks key tiles per CTA,
// accumulates dK/dV for all query heads of its KV group in registers and
// adds dQ with fp32 global reductions.
//
// Forward outputs o [T, Hq*128] and lse [Hq, T] (natural log, scale
// included); backward writes dq/dk/dv into dqkv [T, (Hq + 2 Hkv) * 128].
#include "common.cuh"

#include <cstdlib>

namespace t1 {
namespace attn {

using bf16 = __nv_bfloat16;

constexpr int D = 128;       // head dim
constexpr int BR = 64;       // query rows per tile
constexpr int BC = 64;       // keys per tile
constexpr int ROW_BYTES = D * 2;  // 256
constexpr int TILE_BYTES = 64 * ROW_BYTES;  // 16 KB
constexpr float LOG2E = 1.4426950408889634f;

// 16-byte chunk c (0..15) of row r, XOR-swizzled against bank conflicts.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * ROW_BYTES + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

// Copy a 64 x 128 bf16 tile (rows `ld` elements apart) into swizzled smem.
__device__ __forceinline__ void load_tile(uint32_t smem, const bf16* g, long ld, int tid,
                                          int nthreads) {
  for (int i = tid; i < 64 * 16; i += nthreads) {
    int r = i >> 4, c = i & 15;
    cp_async16(smem + swz(r, c), g + r * ld + c * 8);
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// A fragment (16 x 16) of a row-major smem tile at (row0, col0 in elements).
__device__ __forceinline__ void frag_a(uint32_t base, int row0, int col0, int lane, uint32_t (&a)[4]) {
  int r = row0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  int c = (col0 >> 3) + (lane >> 4);
  ldsm_x4(base + swz(r, c), a[0], a[1], a[2], a[3]);
}

// B fragments for two n-tiles (n0..n0+7, n0+8..n0+15) x k = 16 from a tile
// stored [n][k] row-major (k contiguous): "NT" operand (e.g. K for Q K^T).
__device__ __forceinline__ void frag_b_nt(uint32_t base, int n0, int k0, int lane, uint32_t (&b)[4]) {
  // matrices: (n0..+7, k0..+7), (n0..+7, k0+8..), (n0+8.., k0..), (n0+8.., k0+8..)
  int r = n0 + (lane & 7) + ((lane >> 4) << 3);
  int c = (k0 >> 3) + ((lane >> 3) & 1);
  ldsm_x4(base + swz(r, c), b[0], b[1], b[2], b[3]);
  // b[0], b[1] -> n-tile 0 (k lo, k hi); b[2], b[3] -> n-tile 1
}

// B fragments for two n-tiles x k = 16 from a tile stored [k][n] row-major
// (n contiguous): "NN" operand (e.g. V for P V), via ldmatrix.trans.
__device__ __forceinline__ void frag_b_nn(uint32_t base, int k0, int n0, int lane, uint32_t (&b)[4]) {
  // matrices: (k0..+7, n0..+7), (k0+8.., n0..), (k0.., n0+8..), (k0+8.., n0+8..)
  int r = k0 + (lane & 7) + (((lane >> 3) & 1) << 3);
  int c = (n0 >> 3) + (lane >> 4);
  ldsm_x4_t(base + swz(r, c), b[0], b[1], b[2], b[3]);
}

// ================================================================ forward
// grid (S / 64, Hq, B), 128 threads: warp w owns query rows 16w..16w+15.
__global__ void __launch_bounds__(128) attn_fwd_kernel(const bf16* __restrict__ qkv, long ld,
                                                       bf16* __restrict__ out, long ldo,
                                                       float* __restrict__ lse, int S, int T,
                                                       int Hq, int Hkv, float scale) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const uint32_t sK = sQ + TILE_BYTES;           // 2 buffers
  const uint32_t sV = sK + 2 * TILE_BYTES;       // 2 buffers
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = (gridDim.x - 1) - blockIdx.x;   // heavy (late) tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (Hq / Hkv);
  const long tok0 = static_cast<long>(b) * S;
  // uniform over the CTA: the query tile and the head columns exist
  if (T1_OOB(tok0 + (qt + 1) * BR - 1, T) || T1_OOB((long)(Hq + 2 * Hkv) * D - 1, ld) ||
      T1_OOB((long)Hq * D - 1, ldo))
    return;
  const bf16* q_g = qkv + (tok0 + qt * BR) * ld + h * D;
  const bf16* k_g = qkv + tok0 * ld + (Hq + hk) * D;
  const bf16* v_g = qkv + tok0 * ld + (Hq + Hkv + hk) * D;

  load_tile(sQ, q_g, ld, tid, 128);
  load_tile(sK, k_g, ld, tid, 128);
  load_tile(sV, v_g, ld, tid, 128);
  cp_commit();

  const float sl2 = scale * LOG2E;
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  uint32_t qa[8][4];
  const int n_kv = qt + 1;
  const int g = lane >> 2, t4 = lane & 3;
  const int qrow0 = qt * BR + warp * 16 + g;  // rows qrow0 and qrow0 + 8

  for (int kt = 0; kt < n_kv; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_kv) {
      load_tile(sK + (buf ^ 1) * TILE_BYTES, k_g + (kt + 1) * BC * ld, ld, tid, 128);
      load_tile(sV + (buf ^ 1) * TILE_BYTES, v_g + (kt + 1) * BC * ld, ld, tid, 128);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (kt == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) frag_a(sQ, warp * 16, kk * 16, lane, qa[kk]);
    }
    const uint32_t kb = sK + buf * TILE_BYTES, vb = sV + buf * TILE_BYTES;
    // S = Q K^T : 16 x 64 per warp
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        uint32_t bfr[4];
        frag_b_nt(kb, jp * 16, kk * 16, lane, bfr);
        mma16816(s[2 * jp], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], bfr[0], bfr[1]);
        mma16816(s[2 * jp + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], bfr[2], bfr[3]);
      }
    }
    // scale (base 2) + causal mask on the diagonal tile
    const bool diag = kt == qt;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[j][e] * sl2;
        if (diag) {
          int key = kt * BC + j * 8 + 2 * t4 + (e & 1);
          int row = qrow0 + ((e >> 1) << 3);
          if (key > row) v = -INFINITY;
        }
        s[j][e] = v;
      }
    }
    // online softmax for rows g (e = 0,1) and g + 8 (e = 2,3)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fmaxf(s[j][2 * hr], s[j][2 * hr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mnew = fmaxf(m[hr], mx);
      const float corr = exp2f(m[hr] - mnew);  // m = -inf initially -> 0
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float p0 = exp2f(s[j][2 * hr] - mnew), p1 = exp2f(s[j][2 * hr + 1] - mnew);
        s[j][2 * hr] = p0;
        s[j][2 * hr + 1] = p1;
        rs += p0 + p1;
      }
      l[hr] = l[hr] * corr + rs;
      m[hr] = mnew;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][2 * hr] *= corr;
        o[j][2 * hr + 1] *= corr;
      }
    }
    // O += P V : P (16 x 64) from registers, V tile [key][d]
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16 keys per step
      uint32_t pa0 = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      uint32_t pa1 = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      uint32_t pa2 = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      uint32_t pa3 = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int jp = 0; jp < 8; ++jp) {  // 16 d columns per step
        uint32_t bfr[4];
        frag_b_nn(vb, kk * 16, jp * 16, lane, bfr);
        mma16816(o[2 * jp], pa0, pa1, pa2, pa3, bfr[0], bfr[1]);
        mma16816(o[2 * jp + 1], pa0, pa1, pa2, pa3, bfr[2], bfr[3]);
      }
    }
    __syncthreads();
  }
  // finalize
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float ls = l[hr];
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    const float inv = 1.f / ls;
    const int row = qrow0 + hr * 8;
    bf16* orow = out + (tok0 + row) * ldo + h * D;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      *reinterpret_cast<__nv_bfloat162*>(orow + j * 8 + 2 * t4) =
          __floats2bfloat162_rn(o[j][2 * hr] * inv, o[j][2 * hr + 1] * inv);
    }
    if (t4 == 0) lse[static_cast<long>(h) * T + tok0 + row] = (m[hr] + __log2f(ls)) / LOG2E;
  }
}

// ============================================================== backward
// delta[h, t] = sum_d dO[t, h, d] * O[t, h, d]
__global__ void attn_bwd_delta_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ out,
                                      long ldo, float* __restrict__ delta, int T, int Hq) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= T * Hq) return;
  const int t = w / Hq, h = w % Hq;
  const bf16* a = dout + static_cast<long>(t) * ldo + h * D + lane * 4;
  const bf16* b = out + static_cast<long>(t) * ldo + h * D + lane * 4;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) s += __bfloat162float(a[i]) * __bfloat162float(b[i]);
  s = warp_sum(s);
  if (lane == 0) delta[static_cast<long>(h) * T + t] = s;
}

// grid (S / 64, Hkv, B), 128 threads: warp w owns keys 16w..16w+15 of the
// key tile; loops over the G query heads of the group and over query tiles
// qt >= kt.  dK/dV for the warp's 16 keys stay in registers.
__global__ void __launch_bounds__(128) attn_bwd_kernel(
    const bf16* __restrict__ qkv, long ld, const bf16* __restrict__ dout, long ldo,
    const float* __restrict__ lse, const float* __restrict__ delta, float* __restrict__ dq_acc,
    bf16* __restrict__ dqkv, long ldd, int S, int T, int Hq, int Hkv, float scale) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const uint32_t sV = sK + TILE_BYTES;
  const uint32_t sQ = sV + TILE_BYTES;                // 2 buffers
  const uint32_t sdO = sQ + 2 * TILE_BYTES;           // 2 buffers
  const uint32_t sdS = sdO + 2 * TILE_BYTES;          // [64 keys][64 q] bf16, 128 B rows
  float* s_lse = reinterpret_cast<float*>(smem + 6 * TILE_BYTES + 64 * 128);  // 2 x 64
  float* s_delta = s_lse + 128;                                               // 2 x 64

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kt = blockIdx.x;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int G = Hq / Hkv;
  const long tok0 = static_cast<long>(b) * S;
  const int nq = S / BR;
  const int g = lane >> 2, t4 = lane & 3;
  const float sl2 = scale * LOG2E;
  // uniform over the CTA: the key tile, the sequence and the head columns exist
  if (T1_OOB(tok0 + S - 1, T) || T1_OOB(kt, nq) || T1_OOB((long)(Hq + 2 * Hkv) * D - 1, ld) ||
      T1_OOB((long)(Hq + 2 * Hkv) * D - 1, ldd) || T1_OOB((long)Hq * D - 1, ldo))
    return;

  load_tile(sK, qkv + (tok0 + kt * BC) * ld + (Hq + hk) * D, ld, tid, 128);
  load_tile(sV, qkv + (tok0 + kt * BC) * ld + (Hq + Hkv + hk) * D, ld, tid, 128);
  cp_commit();

  float dk[16][4], dv[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[j][e] = dv[j][e] = 0.f;

  const int n_items = G * (nq - kt);
  auto issue = [&](int item, int buf) {
    const int hh = hk * G + item / (nq - kt);
    const int qt = kt + item % (nq - kt);
    load_tile(sQ + buf * TILE_BYTES, qkv + (tok0 + qt * BR) * ld + hh * D, ld, tid, 128);
    load_tile(sdO + buf * TILE_BYTES, dout + (tok0 + qt * BR) * ldo + hh * D, ldo, tid, 128);
    if (tid < 64) {
      s_lse[buf * 64 + tid] = lse[static_cast<long>(hh) * T + tok0 + qt * BR + tid];
      s_delta[buf * 64 + tid] = delta[static_cast<long>(hh) * T + tok0 + qt * BR + tid];
    }
    cp_commit();
  };
  issue(0, 0);

  for (int it = 0; it < n_items; ++it) {
    const int buf = it & 1;
    const int hh = hk * G + it / (nq - kt);
    const int qt = kt + it % (nq - kt);
    if (it + 1 < n_items) {
      issue(it + 1, buf ^ 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const uint32_t qb = sQ + buf * TILE_BYTES, ob = sdO + buf * TILE_BYTES;
    const float* lse_t = s_lse + buf * 64;
    const float* del_t = s_delta + buf * 64;
    // S^T = K Q^T and dP^T = V dO^T : [16 keys x 64 q] per warp
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[j][e] = dpt[j][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t ka[4], va[4];  // this warp's 16 K / V rows, d = 16kk..16kk+15
      frag_a(sK, warp * 16, kk * 16, lane, ka);
      frag_a(sV, warp * 16, kk * 16, lane, va);
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        uint32_t bq[4], bo[4];
        frag_b_nt(qb, jp * 16, kk * 16, lane, bq);
        frag_b_nt(ob, jp * 16, kk * 16, lane, bo);
        mma16816(st[2 * jp], ka[0], ka[1], ka[2], ka[3], bq[0], bq[1]);
        mma16816(st[2 * jp + 1], ka[0], ka[1], ka[2], ka[3], bq[2], bq[3]);
        mma16816(dpt[2 * jp], va[0], va[1], va[2], va[3], bo[0], bo[1]);
        mma16816(dpt[2 * jp + 1], va[0], va[1], va[2], va[3], bo[2], bo[3]);
      }
    }
    // P^T and dS^T; element (key = kt*64 + 16w + g (+8), q = qt*64 + 8j + 2 t4 (+1))
    const bool diag = qt == kt;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ql = j * 8 + 2 * t4 + (e & 1);
        const int kl = warp * 16 + g + ((e >> 1) << 3);
        float p = exp2f(st[j][e] * sl2 - lse_t[ql] * LOG2E);
        if (diag && kl > ql) p = 0.f;
        st[j][e] = p;
        dpt[j][e] = p * (dpt[j][e] - del_t[ql]);  // dS (without the softmax scale)
      }
    }
    // dV += P^T dO, dK += dS^T Q : A = [16 keys x 64 q] from registers
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa0 = pack_bf16(st[2 * kk][0], st[2 * kk][1]);
      uint32_t pa1 = pack_bf16(st[2 * kk][2], st[2 * kk][3]);
      uint32_t pa2 = pack_bf16(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      uint32_t pa3 = pack_bf16(st[2 * kk + 1][2], st[2 * kk + 1][3]);
      uint32_t da0 = pack_bf16(dpt[2 * kk][0], dpt[2 * kk][1]);
      uint32_t da1 = pack_bf16(dpt[2 * kk][2], dpt[2 * kk][3]);
      uint32_t da2 = pack_bf16(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]);
      uint32_t da3 = pack_bf16(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3]);
#pragma unroll
      for (int jp = 0; jp < 8; ++jp) {
        uint32_t bo[4], bq[4];
        frag_b_nn(ob, kk * 16, jp * 16, lane, bo);
        frag_b_nn(qb, kk * 16, jp * 16, lane, bq);
        mma16816(dv[2 * jp], pa0, pa1, pa2, pa3, bo[0], bo[1]);
        mma16816(dv[2 * jp + 1], pa0, pa1, pa2, pa3, bo[2], bo[3]);
        mma16816(dk[2 * jp], da0, da1, da2, da3, bq[0], bq[1]);
        mma16816(dk[2 * jp + 1], da0, da1, da2, da3, bq[2], bq[3]);
      }
    }
    // stage dS^T [64 keys][64 q] (bf16, 128-byte rows, chunk swizzle) for dQ
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int kl = warp * 16 + g + hr * 8;
        const int ql = j * 8 + 2 * t4;
        const uint32_t addr = sdS + kl * 128 + (((ql >> 3) ^ (kl & 7)) << 4) + (ql & 7) * 2;
        const uint32_t v = pack_bf16(dpt[j][2 * hr], dpt[j][2 * hr + 1]);
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v));
      }
    }
    __syncthreads();
    // dQ[q, :] += sum_key dS[q, key] K[key, :] for the warp's 16 query rows
    {
      float dqv[16][4];
#pragma unroll
      for (int j = 0; j < 16; ++j) dqv[j][0] = dqv[j][1] = dqv[j][2] = dqv[j][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // 16 keys per step
        // A = dS [16 q x 16 keys] from dS^T [key][q] via ldmatrix.trans
        uint32_t a[4];
        {
          const int key = kk * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int qc = (warp * 16 >> 3) + ((lane >> 3) & 1);
          ldsm_x4_t(sdS + key * 128 + ((qc ^ (key & 7)) << 4), a[0], a[1], a[2], a[3]);
        }
#pragma unroll
        for (int jp = 0; jp < 8; ++jp) {
          uint32_t bk[4];
          frag_b_nn(sK, kk * 16, jp * 16, lane, bk);
          mma16816(dqv[2 * jp], a[0], a[1], a[2], a[3], bk[0], bk[1]);
          mma16816(dqv[2 * jp + 1], a[0], a[1], a[2], a[3], bk[2], bk[3]);
        }
      }
      const long qrow = tok0 + qt * BR + warp * 16 + g;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          float* dst = dq_acc + ((qrow + hr * 8) * Hq + hh) * D + j * 8 + 2 * t4;
          atomicAdd(dst, dqv[j][2 * hr] * scale);
          atomicAdd(dst + 1, dqv[j][2 * hr + 1] * scale);
        }
      }
    }
    __syncthreads();
  }
  // write dK, dV (bf16) for the warp's 16 keys
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const long key = tok0 + kt * BC + warp * 16 + g + hr * 8;
    bf16* dkr = dqkv + key * ldd + (Hq + hk) * D;
    bf16* dvr = dqkv + key * ldd + (Hq + Hkv + hk) * D;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      *reinterpret_cast<__nv_bfloat162*>(dkr + j * 8 + 2 * t4) =
          __floats2bfloat162_rn(dk[j][2 * hr] * scale, dk[j][2 * hr + 1] * scale);
      *reinterpret_cast<__nv_bfloat162*>(dvr + j * 8 + 2 * t4) =
          __floats2bfloat162_rn(dv[j][2 * hr], dv[j][2 * hr + 1]);
    }
  }
}

// dq (fp32 [T, Hq, 128]) -> bf16 columns of dqkv
__global__ void attn_dq_convert_kernel(const float* __restrict__ acc, bf16* __restrict__ dqkv,
                                       long ldd, int T, int Hq) {
  const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;  // one per 8 values
  const long n = static_cast<long>(T) * Hq * D / 8;
  if (i >= n) return;
  const long e = i * 8;
  const long t = e / (Hq * D), c = e % (Hq * D);
  const float4* s = reinterpret_cast<const float4*>(acc + e);
  float4 a = s[0], bq = s[1];
  float f[8] = {a.x, a.y, a.z, a.w, bq.x, bq.y, bq.z, bq.w};
  store8(dqkv + t * ldd + c, f);
}

}  // namespace attn

T1_BOUNDS_READER(attention)

// ================================================================ host side
static void check_qkv(const torch::Tensor& qkv, int64_t n_q, int64_t n_kv, int64_t D, int64_t S) {
  T1_CHECK_INPUT(qkv, torch::kBFloat16);
  TORCH_CHECK(D == attn::D, "attention kernels are built for head_dim 128, got ", D);
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.size(1) >= (n_q + 2 * n_kv) * D,
              "qkv must be row-major [T, (n_q + 2 n_kv) D]");
  TORCH_CHECK(n_q % n_kv == 0, "n_q must be a multiple of n_kv");
  TORCH_CHECK(S % 64 == 0 && qkv.size(0) % S == 0, "seq_len must be a multiple of 64 and divide T");
  TORCH_CHECK(qkv.stride(0) % 8 == 0, "qkv row stride must be a multiple of 8");
}

std::vector<torch::Tensor> attention_fwd_tc(torch::Tensor qkv, int64_t n_q, int64_t n_kv, int64_t D,
                                            int64_t S);
std::vector<torch::Tensor> attention_fwd_tc2(torch::Tensor qkv, int64_t n_q, int64_t n_kv, int64_t S);
void attention_bwd_pipe_core(torch::Tensor dout, torch::Tensor qkv, torch::Tensor lse,
                             torch::Tensor delta, torch::Tensor dq_acc, torch::Tensor dqkv, int64_t n_q,
                             int64_t n_kv, int64_t S);
void attention_bwd_tc_core(torch::Tensor dout, torch::Tensor qkv, torch::Tensor lse,
                           torch::Tensor delta, torch::Tensor dq_acc, torch::Tensor dqkv, int64_t n_q,
                           int64_t n_kv, int64_t S);

// Implementation of forward and backward: 0 = mma.sync tiles (this file),
// 1 = tcgen05 with one 128-row query tile per CTA (attention_tc.cu),
// 2 = the two-tile tcgen05 forward (attention_fwd2.cu, the default; it falls
// back to mode 1 when seq_len is not a multiple of 256) with the tcgen05
// backward.  Per process: attn_set_mode() or T1_ATTN_TC=0/1/2.
static int& attn_mode() {
  static int mode = [] {
    const char* e = std::getenv("T1_ATTN_TC");
    if (e != nullptr && (e[0] == '0' || e[0] == '1')) return e[0] - '0';
    return 2;
  }();
  return mode;
}

void attn_set_mode(int64_t mode) {
  TORCH_CHECK(mode >= 0 && mode <= 2, "attention mode must be 0 (mma.sync), 1 or 2 (tcgen05)");
  attn_mode() = static_cast<int>(mode);
}

int64_t attn_get_mode() { return attn_mode(); }

// tcgen05 backward: pipelined (attention_bwd2.cu, the default) or the
// serial one of attention_tc.cu (T1_ATTN_BWD_PIPE=0 / attn_set_bwd_pipelined).
static bool& attn_bwd_pipelined() {
  static bool on = [] {
    const char* e = std::getenv("T1_ATTN_BWD_PIPE");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

void attn_set_bwd_pipelined(bool on) { attn_bwd_pipelined() = on; }

std::vector<torch::Tensor> attention_fwd(torch::Tensor qkv, int64_t n_q, int64_t n_kv, int64_t D,
                                         int64_t S) {
  if (attn_mode() == 2 && S % 256 == 0) {
    check_qkv(qkv, n_q, n_kv, D, S);
    return attention_fwd_tc2(qkv, n_q, n_kv, S);
  }
  if (attn_mode() >= 1) return attention_fwd_tc(qkv, n_q, n_kv, D, S);
  check_qkv(qkv, n_q, n_kv, D, S);
  const int64_t T = qkv.size(0), B = T / S;
  auto out = torch::empty({T, n_q * D}, qkv.options());
  auto lse = torch::empty({n_q, T}, qkv.options().dtype(torch::kFloat32));
  const int smem = 5 * attn::TILE_BYTES;
  static bool cfg = false;
  if (!cfg) {
    T1_CHECK_CUDA(cudaFuncSetAttribute(attn::attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cfg = true;
  }
  dim3 grid(S / attn::BR, n_q, B);
  attn::attn_fwd_kernel<<<grid, 128, smem, stream()>>>(
      (const __nv_bfloat16*)qkv.data_ptr(), qkv.stride(0), (__nv_bfloat16*)out.data_ptr(), out.stride(0),
      lse.data_ptr<float>(), S, T, n_q, n_kv, 1.0f / std::sqrt((float)D));
  check_launch("attention_fwd");
  count_launch();
  return {out, lse};
}

torch::Tensor attention_bwd(torch::Tensor dout, torch::Tensor qkv, torch::Tensor out,
                            torch::Tensor lse, int64_t n_q, int64_t n_kv, int64_t D, int64_t S) {
  check_qkv(qkv, n_q, n_kv, D, S);
  T1_CHECK_INPUT(dout, torch::kBFloat16);
  T1_CHECK_INPUT(out, torch::kBFloat16);
  T1_CHECK_INPUT(lse, torch::kFloat32);
  const int64_t T = qkv.size(0), B = T / S;
  TORCH_CHECK(dout.is_contiguous() && out.is_contiguous() && dout.size(1) == n_q * D &&
                  out.size(1) == n_q * D, "dout/out must be contiguous [T, n_q D]");
  auto dqkv = torch::empty({T, (n_q + 2 * n_kv) * D}, qkv.options());
  auto delta = torch::empty({n_q, T}, qkv.options().dtype(torch::kFloat32));
  auto dq_acc = torch::zeros({T, n_q, D}, qkv.options().dtype(torch::kFloat32));
  {
    const long warps = T * n_q;
    attn::attn_bwd_delta_kernel<<<(warps * 32 + 255) / 256, 256, 0, stream()>>>(
        (const __nv_bfloat16*)dout.data_ptr(), (const __nv_bfloat16*)out.data_ptr(), out.stride(0),
        delta.data_ptr<float>(), T, n_q);
    check_launch("attention_bwd_delta");
  }
  if (attn_mode() >= 1) {
    if (attn_bwd_pipelined())
      attention_bwd_pipe_core(dout, qkv, lse, delta, dq_acc, dqkv, n_q, n_kv, S);
    else
      attention_bwd_tc_core(dout, qkv, lse, delta, dq_acc, dqkv, n_q, n_kv, S);
  } else {
    const int smem = 6 * attn::TILE_BYTES + 64 * 128 + 4 * 64 * 4;
    static bool cfg = false;
    if (!cfg) {
      T1_CHECK_CUDA(cudaFuncSetAttribute(attn::attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      cfg = true;
    }
    dim3 grid(S / attn::BC, n_kv, B);
    attn::attn_bwd_kernel<<<grid, 128, smem, stream()>>>(
        (const __nv_bfloat16*)qkv.data_ptr(), qkv.stride(0), (const __nv_bfloat16*)dout.data_ptr(),
        dout.stride(0), lse.data_ptr<float>(), delta.data_ptr<float>(), dq_acc.data_ptr<float>(),
        (__nv_bfloat16*)dqkv.data_ptr(), dqkv.stride(0), S, T, n_q, n_kv, 1.0f / std::sqrt((float)D));
    check_launch("attention_bwd");
  }
  const long n8 = T * n_q * D / 8;
  attn::attn_dq_convert_kernel<<<(n8 + 255) / 256, 256, 0, stream()>>>(
      dq_acc.data_ptr<float>(), (__nv_bfloat16*)dqkv.data_ptr(), dqkv.stride(0), T, n_q);
  check_launch("attention_dq_convert");
  count_launch(3);
  return dqkv;
}

}  // namespace t1
