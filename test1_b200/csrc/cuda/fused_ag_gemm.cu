// Shard-mode layer fetch fused with the first consuming GEMM (the QKV
// projection), one kernel per layer and rank:
//
//   * 2 gather warps per CTA read this rank's shard of the layer -- from
//     page-locked host memory (the fp32 master, cast to bf16 in registers,
//     or the bf16 shadow), or, in the staged form, from this rank's own unit
//     where the copy engine placed it one layer ahead -- and store it into
//     every peer's pool unit over NVLink (P2P stores; no multicast), then
//     publish per-256-row-block arrival flags in every peer's signal pad;
//   * the tcgen05 GEMM warps (CTA pairs, cta_group::2, by default; single
//     CTAs when the GEMM mode is 0) compute qkv = x * W_qkv^T from the *local* unit:
//     before TMA-loading the B rows of a tile, the producer waits (bounded)
//     for the arrival flags of the ranks that own those rows, then fences
//     the generic-proxy writes for the async proxy.
//
// The kernel returns once every rank's shard has landed in this GPU's unit,
// so later kernels in the stream see the whole layer.
#include "gemm_core.cuh"
#include "gemm_pair.cuh"

namespace t1 {

uint64_t fused_peer_wait_ns();

T1_BOUNDS_READER(fused_ag_gemm)

CUtensorMap make_map(const void* ptr, int64_t inner, int64_t outer, int64_t ld, int box_outer);
torch::Tensor& gemm_error_word();
int64_t gemm_get_mode();

// shards: CPU int64 [world, 2] = (start, end) of every rank's shard of the
// layer (identical on all ranks); host_src is this rank's shard.
void fused_ag_qkv(torch::Tensor x, torch::Tensor unit, int64_t n_rows, torch::Tensor out,
                  torch::Tensor ptrs, torch::Tensor sigs, torch::Tensor shards, int64_t rank,
                  int64_t world, torch::Tensor host_src, c10::optional<torch::Tensor> host_src_lo,
                  int64_t epoch, torch::Tensor counters, c10::optional<torch::Tensor> rope_cos,
                  c10::optional<torch::Tensor> rope_sin, int64_t rope_S, int64_t rope_cols) {
  T1_CHECK_INPUT(x, torch::kBFloat16);
  T1_CHECK_INPUT(unit, torch::kBFloat16);
  T1_CHECK_INPUT(out, torch::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.is_contiguous(), "x must be contiguous [T, K]");
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == n_rows && out.is_contiguous(),
              "out must be contiguous [T, n_rows]");
  TORCH_CHECK(n_rows % 8 == 0 && K % 8 == 0, "n_rows and K must be multiples of 8");
  TORCH_CHECK(unit.numel() >= n_rows * K, "unit smaller than the QKV weight");
  TORCH_CHECK(world >= 1 && world <= gemm::kAgMaxRanks, "world must be 1..8");
  const int64_t n_blocks = (n_rows + gemm::BN - 1) / gemm::BN;
  TORCH_CHECK(n_blocks <= gemm::kAgMaxBlocks, "QKV weight has too many row blocks");
  TORCH_CHECK(shards.device().is_cpu() && shards.scalar_type() == torch::kInt64 &&
                  shards.dim() == 2 && shards.size(0) == world && shards.size(1) == 2,
              "shards must be a CPU int64 [world, 2] table");
  auto sh = shards.accessor<int64_t, 2>();
  const int64_t shard_off = sh[rank][0];
  const int64_t shard_n = sh[rank][1] - sh[rank][0];
  TORCH_CHECK(shard_off % 8 == 0, "shard offset must be a multiple of 8");
  TORCH_CHECK(sh[rank][1] <= unit.numel(), "shard exceeds the unit");
  TORCH_CHECK(ptrs.device().is_cpu() && sigs.device().is_cpu() && ptrs.numel() == world &&
                  sigs.numel() == world, "peer tables must be CPU int64 [world]");
  TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == torch::kInt32 &&
                  counters.numel() >= gemm::kAgMaxBlocks + 1, "counters must be int32 [65] on the GPU");
  const bool split = host_src_lo.has_value() && host_src_lo->defined();
  TORCH_CHECK(split || host_src.scalar_type() == torch::kFloat32 ||
                  host_src.scalar_type() == torch::kBFloat16,
              "host_src must be fp32, bf16, or the high plane of a split master");
  TORCH_CHECK(host_src.numel() >= shard_n && host_src.is_contiguous(), "host_src too small");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(host_src.data_ptr()) % 16 == 0, "host_src misaligned");

  gemm::AgParams ag{};
  auto pa = ptrs.accessor<int64_t, 1>();
  auto sa = sigs.accessor<int64_t, 1>();
  for (int q = 0; q < world; ++q) {
    ag.peer[q] = static_cast<uint64_t>(pa[q]);
    ag.sig[q] = static_cast<uint64_t>(sa[q]);
  }
  TORCH_CHECK(ag.peer[rank] == reinterpret_cast<uint64_t>(unit.data_ptr()),
              "unit must be this rank's symmetric buffer");
  ag.rank = static_cast<int>(rank);
  ag.world = static_cast<int>(world);
  ag.shard_off = shard_off;
  ag.shard_n = shard_n;
  ag.skip_self = 0;
  if (host_src.is_cuda()) {
    // staged form: the shard already sits in this rank's unit
    TORCH_CHECK(host_src.scalar_type() == torch::kBFloat16 && !(host_src_lo.has_value() && host_src_lo->defined()),
                "a device-resident shard source must be bf16");
    TORCH_CHECK(host_src.data_ptr() == static_cast<void*>(static_cast<__nv_bfloat16*>(unit.data_ptr()) + shard_off),
                "a device-resident shard source must be this rank's unit at the shard offset");
    ag.skip_self = 1;
  }
  const void* src = host_src.data_ptr();
  if (host_src.device().is_cpu()) {
    void* d = nullptr;
    T1_CHECK_CUDA(cudaHostGetDevicePointer(&d, host_src.data_ptr(), 0));
    src = d;
  }
  ag.host_src = src;
  ag.host_src_lo = nullptr;
  if (split) {
    TORCH_CHECK(host_src.element_size() == 2 && host_src_lo->element_size() == 2 &&
                    host_src_lo->numel() >= shard_n && host_src_lo->is_contiguous() &&
                    reinterpret_cast<uintptr_t>(host_src_lo->data_ptr()) % 16 == 0,
                "bad split-master low plane");
    void* d = host_src_lo->data_ptr();
    if (host_src_lo->device().is_cpu()) T1_CHECK_CUDA(cudaHostGetDevicePointer(&d, host_src_lo->data_ptr(), 0));
    ag.host_src_lo = d;
    ag.src_kind = 2;
  } else {
    ag.src_kind = host_src.scalar_type() == torch::kFloat32 ? 1 : 0;
  }
  ag.epoch = static_cast<uint32_t>(epoch);
  ag.wait_ns = fused_peer_wait_ns();
  ag.n_blocks = static_cast<int>(n_blocks);
  ag.block_elems = static_cast<long>(gemm::BN) * K;
  // owners of each 256-row block: ranks whose shard intersects its elements
  for (int b = 0; b < n_blocks; ++b) {
    const int64_t lo = static_cast<int64_t>(b) * gemm::BN * K;
    const int64_t hi = std::min<int64_t>(n_rows, static_cast<int64_t>(b + 1) * gemm::BN) * K;
    uint8_t mask = 0;
    for (int q = 0; q < world; ++q)
      if (sh[q][0] < hi && sh[q][1] > lo && sh[q][1] > sh[q][0]) mask |= static_cast<uint8_t>(1u << q);
    ag.owners[b] = mask;
  }
  ag.counters = counters.data_ptr<int>();

  gemm::Params p;
  p.M = M;
  p.N = n_rows;
  p.K = K;
  p.C = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldc = out.stride(0);
  p.R = nullptr;
  p.ldr = 0;
  p.k_blocks = (K + gemm::BK - 1) / gemm::BK;
  p.err = gemm_error_word().data_ptr<int>();
  p.rope_cos = p.rope_sin = nullptr;
  p.rope_S = 1;
  p.rope_cols = 0;
  // RoPE in the epilogue (TMA-store mode only; otherwise the caller rotates)
  const bool rope = rope_cos.has_value() && rope_cos->defined() && rope_cols > 0;
  if (rope) {
    TORCH_CHECK(gemm_get_mode() == 2, "the fused RoPE epilogue needs GEMM mode 2");
    TORCH_CHECK(rope_sin.has_value() && rope_sin->defined() && rope_cos->scalar_type() == torch::kFloat32 &&
                    rope_cos->is_cuda() && rope_cos->is_contiguous() && rope_sin->is_contiguous() &&
                    rope_cos->dim() == 2 && rope_cos->size(1) == 64 && rope_cos->size(0) >= rope_S &&
                    rope_sin->sizes() == rope_cos->sizes() && rope_S > 0,
                "rope tables must be contiguous fp32 [>= S, 64]");
    TORCH_CHECK(rope_cols % 128 == 0 && rope_cols <= n_rows, "rope_cols must be whole heads");
    p.rope_cos = rope_cos->data_ptr<float>();
    p.rope_sin = rope_sin->data_ptr<float>();
    p.rope_S = static_cast<int>(rope_S);
    p.rope_cols = static_cast<int>(rope_cols);
  }
  if (gemm_get_mode() >= 1) {
    // CTA pairs: 256 x 256 tiles, the B row blocks match the arrival flags
    p.tiles_m = (M + gemm::PAIR_BM - 1) / gemm::PAIR_BM;
    p.tiles_n = (n_rows + gemm::PAIR_BN - 1) / gemm::PAIR_BN;
    p.num_tiles = p.tiles_m * p.tiles_n;
    CUtensorMap ta = make_map(x.data_ptr(), K, M, x.stride(0), gemm::PAIR_HALF);
    CUtensorMap tb = make_map(unit.data_ptr(), K, n_rows, K, gemm::PAIR_HALF);
    // every CTA gathers, so the grid spans all SMs even when tiles are few
    const int clusters = num_sms() / 2;
    if (gemm_get_mode() == 2 && rope) {
      CUtensorMap tc = make_map(out.data_ptr(), n_rows, M, out.stride(0), 32);
      auto kern = gemm::gemm_pair_kernel<false, false, gemm::kStore, true, true, true>;
      static bool rope_configured = false;
      if (!rope_configured) {
        T1_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           gemm::PAIR_SMEM_BYTES_TMA));
        rope_configured = true;
      }
      kern<<<2 * clusters, 256, gemm::PAIR_SMEM_BYTES_TMA, stream()>>>(ta, tb, p, ag, tc, tc);
    } else if (gemm_get_mode() == 2) {
      CUtensorMap tc = make_map(out.data_ptr(), n_rows, M, out.stride(0), 32);
      auto kern = gemm::gemm_pair_kernel<false, false, gemm::kStore, true, true>;
      static bool tma_configured = false;
      if (!tma_configured) {
        T1_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           gemm::PAIR_SMEM_BYTES_TMA));
        tma_configured = true;
      }
      kern<<<2 * clusters, 256, gemm::PAIR_SMEM_BYTES_TMA, stream()>>>(ta, tb, p, ag, tc, tc);
    } else {
      auto kern = gemm::gemm_pair_kernel<false, false, gemm::kStore, true, false>;
      static bool pair_configured = false;
      if (!pair_configured) {
        T1_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           gemm::PAIR_SMEM_BYTES));
        pair_configured = true;
      }
      kern<<<2 * clusters, 256, gemm::PAIR_SMEM_BYTES, stream()>>>(ta, tb, p, ag, ta, ta);
    }
    check_launch("fused_ag_qkv (pair)");
    count_launch();
    return;
  }
  TORCH_CHECK(!rope, "the fused RoPE epilogue needs the CTA-pair GEMM");
  p.tiles_m = (M + gemm::BM - 1) / gemm::BM;
  p.tiles_n = (n_rows + gemm::BN - 1) / gemm::BN;
  p.num_tiles = p.tiles_m * p.tiles_n;
  CUtensorMap ta = make_map(x.data_ptr(), K, M, x.stride(0), gemm::BM);
  CUtensorMap tb = make_map(unit.data_ptr(), K, n_rows, K, gemm::BN);
  auto kern = gemm::gemm_bf16_kernel<false, false, gemm::kStore, true>;
  static bool configured = false;
  if (!configured) {
    T1_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       gemm::SMEM_BYTES));
    configured = true;
  }
  const int grid = std::min(p.num_tiles, num_sms());
  kern<<<grid, 256, gemm::SMEM_BYTES, stream()>>>(ta, tb, p, ag);
  check_launch("fused_ag_qkv");
  count_launch();
}

}  // namespace t1
