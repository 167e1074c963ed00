// Persistent bf16 GEMM on the 5th-generation tensor cores (tcgen05) for
// sm_100a.
//
//   C[M, N] (bf16, row stride ldc) = A[M, K] * B[N, K]^T  (+ R[M, N])
//
// A and B are each either K-major (rows contiguous along K) or MN-major
// (stored transposed, contiguous along M / N), which covers the three
// products of a linear layer without any transpose copies:
//   forward  y  = x  W^T : A = x  [T, K] K-major,    B = W [N, K] K-major
//   dgrad    dx = dy W   : A = dy [T, N] K-major,    B = W stored [N, K] -> MN-major
//   wgrad    dW = dy^T x : A = dy stored [T, N] -> MN-major, B = x stored [T, K] -> MN-major
//
// Structure (one CTA per SM, 192 threads, warp-specialised):
//   warp 0     TMA producer: 128B-swizzled tiles of A (128 x 64) and B
//              (256 x 64) into a 4-stage shared-memory ring, completion
//              tracked by mbarriers (byte counts).  No multicast.
//   warp 1     allocates 512 TMEM columns; one thread issues
//              tcgen05.mma (M=128, N=256, K=16) into one of two 128x256 fp32
//              TMEM accumulators and commits stage-release / tile-ready
//              barriers.
//   warps 2-5  epilogue: tcgen05.ld the finished accumulator (each warp owns
//              its 32-lane TMEM quarter = 32 rows), optional residual add,
//              bf16 rounding, 16-byte global stores; then hand the
//              accumulator back, so tile i's epilogue overlaps tile i+1's
//              MMAs.
// Tiles are visited in grouped (GROUP_M) raster order for L2 reuse.  All
// barrier waits are bounded (see sm100.cuh); a timeout writes a code to the
// error word and the CTA unwinds.
//
// Pair mode (gemm_pair.cuh, cta_group::2): CTA pairs compute 256 x 256
// tiles with one MMA stream, each CTA staging half of the operands.  The
// mode is chosen per process: gemm_set_mode(0 = single CTA, 1 = pairs with
// register-store epilogue, 2 = pairs with shared-memory + TMA-store
// epilogue), or the environment variable T1_GEMM_MODE (T1_GEMM_PAIR=0 still
// selects the single-CTA kernel).
#include "gemm_core.cuh"
#include "gemm_pair.cuh"

#include <cstdlib>

namespace t1 {

// GEMM mode when neither T1_GEMM_MODE nor T1_GEMM_PAIR is set.
constexpr int kDefaultGemmMode = 2;

// ================================================================ host side
T1_BOUNDS_READER(gemm)

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    T1_CHECK_CUDA(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                                   cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr != nullptr,
                "cuTensorMapEncodeTiled not available from the driver");
    return reinterpret_cast<EncodeTiledFn>(ptr);
  }();
  return fn;
}

// 2-D bf16 tensor map, 128B swizzle: `inner` contiguous elements per row,
// `outer` rows, `ld` elements between rows, box = 64 x box_outer.
CUtensorMap make_map(const void* ptr, int64_t inner, int64_t outer, int64_t ld,
                            int box_outer) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "GEMM operand must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "GEMM operand row stride must be a multiple of 8 elements");
  TORCH_CHECK(inner % 8 == 0, "GEMM operand contiguous extent must be a multiple of 8");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with ", (int)r);
  return m;
}

// 2-D fp32 tensor map, 128B swizzle, box = 32 x 32 (one 128-byte row per
// box row): `inner` contiguous elements per row, `outer` rows, `ld` elements
// between rows.  Used for bulk reduce-adds into fp32 accumulators.
CUtensorMap make_map_f32(const void* ptr, int64_t inner, int64_t outer, int64_t ld) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "fp32 tensor must be 16-byte aligned");
  TORCH_CHECK((ld * 4) % 16 == 0 && inner % 32 == 0, "fp32 rows must be multiples of 32 elements");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 4)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(ptr), dims, strides,
                           box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (fp32) failed with ", (int)r);
  return m;
}

torch::Tensor& gemm_error_word() {
  static thread_local std::unordered_map<int, torch::Tensor> words;
  int dev = 0;
  cudaGetDevice(&dev);
  auto it = words.find(dev);
  if (it == words.end()) {
    auto t = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, dev));
    it = words.emplace(dev, t).first;
  }
  return it->second;
}

static int& gemm_mode() {
  static int mode = [] {
    const char* m = std::getenv("T1_GEMM_MODE");
    if (m != nullptr && m[0] >= '0' && m[0] <= '2' && m[1] == 0) return m[0] - '0';
    const char* e = std::getenv("T1_GEMM_PAIR");
    return (e != nullptr && e[0] == '0') ? 0 : kDefaultGemmMode;
  }();
  return mode;
}

void gemm_set_mode(int64_t mode) {
  TORCH_CHECK(mode >= 0 && mode <= 2,
              "GEMM mode must be 0 (single CTA), 1 (CTA pairs) or 2 (CTA pairs, TMA-store epilogue)");
  gemm_mode() = static_cast<int>(mode);
}

int64_t gemm_get_mode() { return gemm_mode(); }

// Stream-K tail of the TMA-store pair kernel: on by default, T1_GEMM_STREAMK=0
// or gemm_set_streamk(false) turns it off.
static bool& streamk_on() {
  static bool on = [] {
    const char* e = std::getenv("T1_GEMM_STREAMK");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

void gemm_set_streamk(bool on) { streamk_on() = on; }

// Partial-sum workspace and arrival counters of the stream-K tail, one per
// (device, stream), so GEMMs on different streams never share one; grown on
// demand (the counters are zeroed once and reset by the kernel after use).
struct SkWorkspace {
  torch::Tensor ws, flags;
};

static SkWorkspace& sk_workspace(size_t floats, int flag_ints) {
  static std::unordered_map<uint64_t, SkWorkspace> all;
  int dev = 0;
  cudaGetDevice(&dev);
  const cudaStream_t st = stream();
  const uint64_t key = (static_cast<uint64_t>(dev) << 56) ^ reinterpret_cast<uint64_t>(st);
  SkWorkspace& w = all[key];
  const auto opts = torch::TensorOptions().device(torch::kCUDA, dev);
  if (!w.ws.defined() || static_cast<size_t>(w.ws.numel()) < floats)
    w.ws = torch::empty({static_cast<int64_t>(floats)}, opts.dtype(torch::kFloat32));
  if (!w.flags.defined() || w.flags.numel() < flag_ints)
    w.flags = torch::zeros({flag_ints}, opts.dtype(torch::kInt32));
  return w;
}

// Splits the last, partial wave of tiles along K when a cluster is free for
// each half: with C clusters and R = num_tiles % C tail tiles (2 R <= C),
// each tail tile becomes two pieces of >= 8 k-blocks in the same wave.  Only
// for grids of fewer than 5 waves, where the partial wave is a large share
// of the time (measured: the 256-tile Llama-8B projections gain 6-8 %; grids
// of 12-24 waves showed no gain).
static void plan_streamk(gemm::Params& p, int clusters) {
  p.sk_split = 1;
  p.sk_tail0 = 0;
  p.num_units = p.num_tiles;
  if (!streamk_on()) return;
  const int R = p.num_tiles % clusters;
  if (R == 0 || 2 * R > clusters || p.k_blocks < 16 || p.num_tiles >= 5 * clusters) return;
  p.sk_split = 2;
  p.sk_tail0 = p.num_tiles - R;
  p.num_units = p.sk_tail0 + 2 * R;
  SkWorkspace& w = sk_workspace(static_cast<size_t>(R) * gemm::kSkPartFloats, R * 8);
  p.sk_ws = w.ws.data_ptr<float>();
  p.sk_flags = w.flags.data_ptr<int>();
}

template <bool A_MN, bool B_MN, int EPI, bool TMA_EPI, bool ROPE = false>
static void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, gemm::Params& p,
                        const CUtensorMap& tc, const CUtensorMap& tr) {
  auto kern = gemm::gemm_pair_kernel<A_MN, B_MN, EPI, false, TMA_EPI, ROPE>;
  constexpr int smem = TMA_EPI ? gemm::PAIR_SMEM_BYTES_TMA : gemm::PAIR_SMEM_BYTES;
  static bool configured = false;
  if (!configured) {
    T1_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured = true;
  }
  if (TMA_EPI) plan_streamk(p, num_sms() / 2);
  else {
    p.sk_split = 1;
    p.num_units = p.num_tiles;
  }
  const int clusters = std::min(p.num_units, num_sms() / 2);
  gemm::AgParams none{};
  kern<<<2 * clusters, 192, smem, stream()>>>(ta, tb, p, none, tc, tr);
  check_launch("gemm_bf16 (pair)");
  count_launch();
}

template <bool A_MN, bool B_MN, int EPI>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, gemm::Params& p,
                   const CUtensorMap& tc, const CUtensorMap& tr) {
  if (gemm_mode() == 1) return launch_pair<A_MN, B_MN, EPI, false>(ta, tb, p, tc, tr);
  if (gemm_mode() == 2) return launch_pair<A_MN, B_MN, EPI, true>(ta, tb, p, tc, tr);
  auto kern = gemm::gemm_bf16_kernel<A_MN, B_MN, EPI, false>;
  static bool configured = false;
  if (!configured) {
    T1_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       gemm::SMEM_BYTES));
    configured = true;
  }
  const int grid = std::min(p.num_tiles, num_sms());
  gemm::AgParams none{};
  kern<<<grid, 192, gemm::SMEM_BYTES, stream()>>>(ta, tb, p, none);
  check_launch("gemm_bf16");
  count_launch();
}

// C = A * B^T (+ R).  Logical shapes: A [M, K], B [N, K].  `a_mn` /
// `b_mn` say the operand is stored transposed ([K, M] / [K, N], row-major).
void gemm_bf16(torch::Tensor A, torch::Tensor B, torch::Tensor C, bool a_mn, bool b_mn,
               c10::optional<torch::Tensor> R) {
  T1_CHECK_INPUT(A, torch::kBFloat16);
  T1_CHECK_INPUT(B, torch::kBFloat16);
  T1_CHECK_INPUT(C, torch::kBFloat16);
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "2-D operands expected");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "row-major operands expected");
  const int64_t M = a_mn ? A.size(1) : A.size(0);
  const int64_t K = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0);
  const int64_t KB = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(K == KB, "GEMM reduction extents differ: ", K, " vs ", KB);
  TORCH_CHECK(C.size(0) == M && C.size(1) == N, "C must be [", M, ", ", N, "]");
  TORCH_CHECK(N % 8 == 0 && (C.stride(0) % 8) == 0, "N and ldc must be multiples of 8");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0, "C must be 16-byte aligned");
  if (M == 0 || N == 0) return;
  if (K == 0) {
    if (R.has_value() && R->defined()) C.copy_(*R);
    else C.zero_();
    return;
  }
  const bool pair = gemm_mode() >= 1;
  CUtensorMap ta = a_mn ? make_map(A.data_ptr(), M, K, A.stride(0), 64)
                        : make_map(A.data_ptr(), K, M, A.stride(0), pair ? gemm::PAIR_HALF : gemm::BM);
  CUtensorMap tb = b_mn ? make_map(B.data_ptr(), N, K, B.stride(0), 64)
                        : make_map(B.data_ptr(), K, N, B.stride(0), pair ? gemm::PAIR_HALF : gemm::BN);
  const int tile_m = pair ? gemm::PAIR_BM : gemm::BM;
  const int tile_n = pair ? gemm::PAIR_BN : gemm::BN;
  gemm::Params p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = reinterpret_cast<bf16*>(C.data_ptr());
  p.ldc = C.stride(0);
  p.R = nullptr;
  p.ldr = 0;
  p.tiles_m = (M + tile_m - 1) / tile_m;
  p.tiles_n = (N + tile_n - 1) / tile_n;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.k_blocks = (K + gemm::BK - 1) / gemm::BK;
  p.err = gemm_error_word().data_ptr<int>();
  p.rope_cos = p.rope_sin = nullptr;
  p.rope_S = 1;
  p.rope_cols = 0;
  const bool add = R.has_value() && R->defined();
  if (add) {
    T1_CHECK_INPUT(*R, torch::kBFloat16);
    TORCH_CHECK(R->size(0) == M && R->size(1) == N && R->stride(1) == 1, "residual must be [M, N]");
    TORCH_CHECK(R->stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(R->data_ptr()) % 16 == 0,
                "residual must be 16-byte aligned rows");
    p.R = reinterpret_cast<const bf16*>(R->data_ptr());
    p.ldr = R->stride(0);
  }
  // output / residual maps of the TMA-store epilogue: 64 x 32 boxes
  CUtensorMap tc{}, tr{};
  if (gemm_mode() == 2) {
    tc = make_map(C.data_ptr(), N, M, C.stride(0), 32);
    tr = add ? make_map(R->data_ptr(), N, M, R->stride(0), 32) : tc;
  }
  if (!a_mn && !b_mn) {
    if (add) launch<false, false, gemm::kAddResidual>(ta, tb, p, tc, tr);
    else launch<false, false, gemm::kStore>(ta, tb, p, tc, tr);
  } else if (!a_mn && b_mn) {
    TORCH_CHECK(!add, "residual epilogue is built for the forward and wgrad layouts");
    launch<false, true, gemm::kStore>(ta, tb, p, tc, tr);
  } else if (a_mn && b_mn) {
    // wgrad; with R == C it accumulates (the chunked linear cross-entropy
    // sums its weight gradient over token chunks this way)
    if (add) launch<true, true, gemm::kAddResidual>(ta, tb, p, tc, tr);
    else launch<true, true, gemm::kStore>(ta, tb, p, tc, tr);
  } else {
    TORCH_CHECK(!add, "residual epilogue is built for the forward and wgrad layouts");
    launch<true, false, gemm::kStore>(ta, tb, p, tc, tr);
  }
}

// C = A B^T with the rotary embedding applied to columns [0, rope_cols) in
// the epilogue (the QKV projection: q and k heads of head_dim 128 first).
// A [M, K] and B [N, K] K-major; cos/sin fp32 [>= S, 64]; row r has position
// r % S.  Needs the TMA-store epilogue (GEMM mode 2).
void gemm_bf16_rope(torch::Tensor A, torch::Tensor B, torch::Tensor C, torch::Tensor cos_t,
                    torch::Tensor sin_t, int64_t S, int64_t rope_cols) {
  TORCH_CHECK(gemm_mode() == 2, "the RoPE epilogue needs GEMM mode 2 (TMA-store epilogue)");
  T1_CHECK_INPUT(A, torch::kBFloat16);
  T1_CHECK_INPUT(B, torch::kBFloat16);
  T1_CHECK_INPUT(C, torch::kBFloat16);
  T1_CHECK_INPUT(cos_t, torch::kFloat32);
  T1_CHECK_INPUT(sin_t, torch::kFloat32);
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1 &&
                  C.stride(1) == 1, "row-major 2-D operands expected");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K && C.size(0) == M && C.size(1) == N, "shapes: A [M, K], B [N, K], C [M, N]");
  TORCH_CHECK(N % 8 == 0 && C.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0,
              "C must have 16-byte aligned rows");
  TORCH_CHECK(S > 0 && cos_t.is_contiguous() && sin_t.is_contiguous() && cos_t.dim() == 2 &&
                  cos_t.size(1) == 64 && cos_t.size(0) >= S && sin_t.sizes() == cos_t.sizes(),
              "rope tables must be contiguous fp32 [>= S, 64] (head_dim 128)");
  TORCH_CHECK(rope_cols >= 0 && rope_cols % 128 == 0 && rope_cols <= N, "rope_cols must be whole heads");
  if (M == 0 || N == 0) return;
  TORCH_CHECK(K > 0, "K must be positive");
  CUtensorMap ta = make_map(A.data_ptr(), K, M, A.stride(0), gemm::PAIR_HALF);
  CUtensorMap tb = make_map(B.data_ptr(), K, N, B.stride(0), gemm::PAIR_HALF);
  CUtensorMap tc = make_map(C.data_ptr(), N, M, C.stride(0), 32);
  gemm::Params p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = reinterpret_cast<bf16*>(C.data_ptr());
  p.ldc = C.stride(0);
  p.R = nullptr;
  p.ldr = 0;
  p.tiles_m = (M + gemm::PAIR_BM - 1) / gemm::PAIR_BM;
  p.tiles_n = (N + gemm::PAIR_BN - 1) / gemm::PAIR_BN;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.k_blocks = (K + gemm::BK - 1) / gemm::BK;
  p.err = gemm_error_word().data_ptr<int>();
  p.rope_cos = cos_t.data_ptr<float>();
  p.rope_sin = sin_t.data_ptr<float>();
  p.rope_S = static_cast<int>(S);
  p.rope_cols = static_cast<int>(rope_cols);
  launch_pair<false, false, gemm::kStore, true, true>(ta, tb, p, tc, tc);
}

int64_t gemm_check_error(bool reset) {
  auto& w = gemm_error_word();
  int64_t v = w.item<int>();
  if (reset) w.zero_();
  return v;
}

}  // namespace t1
