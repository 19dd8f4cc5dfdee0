// q3s_head.cu -- q3s_head_sample: the codec head GEMM (q3s_head.cuh) and the
// sampler launched behind it as a programmatic dependent.  A translation unit
// of its own (it needs the driver API's tensor-map types).
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>

#include "q3s_args.cuh"
#include "q3s_head.cuh"
#include "q3s_sampler.h"

namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library); resolved once, racing first callers store the
// same pointer.
EncodeTiled encode_tiled() {
  static std::atomic<EncodeTiled> fn{nullptr};
  EncodeTiled f = fn.load(std::memory_order_acquire);
  if (!f) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    f = reinterpret_cast<EncodeTiled>(p);
    fn.store(f, std::memory_order_release);
  }
  return f;
}

// 2-D bf16 tensor [rows, cols] (row stride `ld` elements), boxes of
// [box_rows, 64] in the 128-byte swizzle; rows past the tensor read as zeros.
bool make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeTiled enc = encode_tiled();
  if (!enc) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(q3s::HEAD_BK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int KS, int BN>
cudaError_t launch_head(const CUtensorMap& th, const CUtensorMap& tw, const q3s::HeadArgs& a, int mtiles,
                        cudaStream_t st) {
  using Tile = q3s::HeadTile<KS, BN>;
  auto kern = q3s::head_gemm_kernel<KS, BN>;
  static std::atomic<uint64_t> attr_done{0};  // per device: the shared-memory opt-in is set
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0ull;
  if (!bit || !(attr_done.load(std::memory_order_acquire) & bit)) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Tile::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(bit, std::memory_order_release);
  }
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(a.V / BN, KS, mtiles);
  lc.blockDim = dim3(q3s::HEAD_NT);
  lc.dynamicSmemBytes = Tile::SMEM_BYTES;
  lc.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = KS;
  at[0].val.clusterDim.z = 1;
  lc.attrs = at;
  lc.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&lc, kern, th, tw, a);
  return e != cudaSuccess ? e : cudaGetLastError();
}

// Clusters of one configuration that can be resident at once (cached per
// device; racing first callers store the same value).
template <int KS, int BN>
int max_active_clusters() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    using Tile = q3s::HeadTile<KS, BN>;
    auto kern = q3s::head_gemm_kernel<KS, BN>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Tile::SMEM_BYTES);
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(1, KS, 1);
    lc.blockDim = dim3(q3s::HEAD_NT);
    lc.dynamicSmemBytes = Tile::SMEM_BYTES;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = KS;
    at[0].val.clusterDim.z = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &lc) != cudaSuccess || n <= 0) n = q3s::sm_count() / KS;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// The configurations, in order of preference: the 4-CTA split (a smaller
// partial tile on the cluster network) from the narrowest tile up (more CTAs,
// fewer bytes each), then the 8-CTA split.
struct HeadCfg {
  int ks, bn;
};
constexpr HeadCfg kHeadCfgs[] = {{4, 64}, {4, 96}, {4, 128}, {8, 128}, {8, 192}};

int max_active(const HeadCfg& c) {
  if (c.ks == 4) return c.bn == 64 ? max_active_clusters<4, 64>() : c.bn == 96 ? max_active_clusters<4, 96>()
                                                                               : max_active_clusters<4, 128>();
  return c.bn == 128 ? max_active_clusters<8, 128>() : max_active_clusters<8, 192>();
}

// The first configuration (in preference order) that divides the problem and
// whose grid is one wave: at most one CTA per SM and every cluster resident;
// without one, the dividing configuration with the fewest CTAs.
bool pick_cfg(int H, int V, int mtiles, HeadCfg& out) {
  bool have = false;
  long fewest = 0;
  for (const HeadCfg& c : kHeadCfgs) {
    if (V % c.bn || H % (c.ks * q3s::HEAD_BK)) continue;
    const long clusters = static_cast<long>(V / c.bn) * mtiles;
    if (clusters * c.ks <= q3s::sm_count() && clusters <= max_active(c)) {
      out = c;
      return true;
    }
    if (!have || clusters * c.ks < fewest) {
      have = true;
      fewest = clusters * c.ks;
      out = c;
    }
  }
  return have;
}
}  // namespace

extern "C" q3s_status q3s_head_sample(const q3s_head_desc* d, void* stream) {
  using q3s::report;
  if (!d) return report(Q3S_ERR_INVALID_ARGUMENT, "q3s_head_sample: desc is NULL");
  if (d->struct_size != sizeof(q3s_head_desc))
    return report(Q3S_ERR_INVALID_ARGUMENT, "q3s_head_sample: struct_size %u != %u (ABI mismatch)", d->struct_size,
                  static_cast<unsigned>(sizeof(q3s_head_desc)));
  const int B = d->batch, H = d->hidden_size, V = d->vocab;
  if (B < 0) return report(Q3S_ERR_INVALID_ARGUMENT, "q3s_head_sample: batch %d < 0", B);
  if (H <= 0 || H % 256 != 0)
    return report(Q3S_ERR_INVALID_ARGUMENT, "q3s_head_sample: hidden_size %d is not a positive multiple of 256", H);
  if (V <= 0 || V % 64 != 0 || V > Q3S_MAX_VOCAB)
    return report(Q3S_ERR_INVALID_ARGUMENT, "q3s_head_sample: vocab %d is not a positive multiple of 64 up to %d", V,
                  Q3S_MAX_VOCAB);
  if (B == 0) return report(Q3S_OK, "");
  if (!d->hidden || !d->weight || !d->logits)
    return report(Q3S_ERR_INVALID_ARGUMENT, "q3s_head_sample: hidden, weight and logits are required");
  if (!aligned16(d->hidden) || !aligned16(d->weight) || !aligned16(d->logits))
    return report(Q3S_ERR_INVALID_ARGUMENT, "q3s_head_sample: hidden, weight and logits must be 16-byte aligned");
  if (d->hidden_row_stride < H || d->hidden_row_stride % 8 || d->weight_row_stride < H ||
      d->weight_row_stride % 8 || d->logits_row_stride < V || d->logits_row_stride % 8)
    return report(Q3S_ERR_INVALID_ARGUMENT,
                  "q3s_head_sample: row strides must be multiples of 8 elements, >= H (hidden, weight) / >= V (logits)");
  const int mtiles = (B + q3s::HEAD_BM - 1) / q3s::HEAD_BM;
  HeadCfg cfg{0, 0};
  if (!pick_cfg(H, V, mtiles, cfg))
    return report(Q3S_ERR_UNSUPPORTED, "q3s_head_sample: no tile configuration for hidden_size %d, vocab %d", H, V);
  CUtensorMap tm_hidden, tm_weight;
  if (!make_map(&tm_hidden, d->hidden, B, H, d->hidden_row_stride, q3s::HEAD_BM) ||
      !make_map(&tm_weight, d->weight, V, H, d->weight_row_stride, cfg.bn))
    return report(Q3S_ERR_CUDA, "q3s_head_sample: cuTensorMapEncodeTiled failed or is unavailable");

  q3s::HeadArgs a;
  a.B = B;
  a.H = H;
  a.V = V;
  a.kchunks = H / (cfg.ks * q3s::HEAD_BK);
  a.logits = static_cast<uint16_t*>(d->logits);
  a.ldl = d->logits_row_stride;
  a.error_word = d->error_word;

  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (cfg.ks == 4)
    e = cfg.bn == 64 ? launch_head<4, 64>(tm_hidden, tm_weight, a, mtiles, st)
      : cfg.bn == 96 ? launch_head<4, 96>(tm_hidden, tm_weight, a, mtiles, st)
                     : launch_head<4, 128>(tm_hidden, tm_weight, a, mtiles, st);
  else
    e = cfg.bn == 128 ? launch_head<8, 128>(tm_hidden, tm_weight, a, mtiles, st)
                      : launch_head<8, 192>(tm_hidden, tm_weight, a, mtiles, st);
  if (e != cudaSuccess) return report(Q3S_ERR_CUDA, "q3s_head_sample: head launch failed: %s", cudaGetErrorString(e));
  if (!d->sample) return report(Q3S_OK, "");

  q3s_sample_desc sd;
  std::memcpy(&sd, d->sample, sizeof(sd));
  if (sd.struct_size != sizeof(q3s_sample_desc))
    return report(Q3S_ERR_INVALID_ARGUMENT, "q3s_head_sample: sample->struct_size %u != %u (ABI mismatch)",
                  sd.struct_size, static_cast<unsigned>(sizeof(q3s_sample_desc)));
  sd.batch = B;
  sd.vocab = V;
  sd.logits = d->logits;
  sd.logits_dtype = Q3S_DTYPE_BF16;
  sd.logits_row_stride = d->logits_row_stride;
  return q3s::sample_impl(&sd, st, true);
}
