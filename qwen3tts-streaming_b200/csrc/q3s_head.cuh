// q3s_head.cuh -- the codec head on the tensor cores: logits = hidden @ W^T
// (bf16 in, fp32 accumulation, bf16 out), the talker's codec_head
// (scripts/export/talker_unified_modules.py:345, nn.Linear(hidden, vocab)) or a
// code-predictor lm_head (scripts/export/utils.py:1223), ahead of the sampler.
//
// Shape of the work at the engine's sizes: B ~ 128 rows, H = 2048, V = 3072.
// The weights (12.6 MB) dominate the bytes and the rows are few, so every SM
// must take a slice of W and read it once: one CTA computes a 128-row x BN-
// vocabulary tile over 1/KS of the hidden dimension (split-K), and the KS
// CTAs of a cluster -- one per K slice -- add their partial tiles through
// distributed shared memory in a fixed order (so the sums are reproducible),
// each CTA finishing 128 / KS of the 128 rows.  The split costs a partial tile
// per CTA on the cluster's network, so KS = 4 where it fills the GPU: for
// V = 3072, BN = 96 and 32 x 4 = 128 CTAs per 128 rows, 224 KB of operands
// and a 48 KB partial tile each (KS = 8 and BN up to 256 for other shapes).
//
// Per CTA (128 threads):
//   warp 0 lane 0   TMA producer: 2-D tiled loads (cp.async.bulk.tensor, no
//                   multicast) of the hidden tile [128 x 64] and the weight
//                   tile [256 x 64] per K chunk into a 4-stage ring, 128-byte
//                   swizzled (the layout the MMA descriptors below name);
//   warp 1 lane 0   MMA issuer: tcgen05.mma.cta_group::1.kind::f16 (bf16 x
//                   bf16 -> fp32), M = 128, N = 256, K = 16 per instruction,
//                   accumulator in TMEM (256 columns); tcgen05.commit frees a
//                   stage and finally signals the epilogue;
//   all 4 warps     epilogue: a cluster barrier (every CTA is past its MMAs,
//                   so every ring can receive); tcgen05.ld of their 32 TMEM
//                   lanes (rows), each row stored straight into the ring of
//                   the CTA that finishes it (st.shared::cluster, slot = this
//                   CTA's K slice); a cluster barrier; the fixed-order sum of
//                   the 8 slices from local shared memory, rounded to bf16.
//
// Every mbarrier wait is bounded; a wait that gives up sets
// Q3S_DEVERR_WAIT_TIMEOUT, waits (bounded) for this CTA's own copies and MMAs,
// still takes both cluster barriers (so no CTA of the cluster waits for it in
// vain) and frees its TMEM.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "q3s_device.cuh"
#include "q3s_sampler.h"

namespace q3s {

constexpr int HEAD_BM = 128;      // rows per tile (MMA M)
constexpr int HEAD_BK = 64;       // K per chunk: one 128-byte swizzled row of bf16
constexpr int HEAD_STAGES = 4;
constexpr int HEAD_NT = 128;
constexpr int HEAD_A_BYTES = HEAD_BM * HEAD_BK * 2;   // 16 KB

// One configuration: KS CTAs per cluster (one K slice each, 4 or 8) and a
// vocabulary tile of BN entries (the MMA's N).
template <int KS, int BN>
struct HeadTile {
  static constexpr int ROWS = HEAD_BM / KS;                     // rows each CTA of a cluster finishes
  static constexpr int TMEM_COLS = BN <= 128 ? 128 : 256;       // power of two >= BN
  static constexpr int B_BYTES = BN * HEAD_BK * 2;
  static constexpr int STAGE_BYTES = HEAD_A_BYTES + B_BYTES;   // multiple of 1024
  static constexpr int RING_BYTES = HEAD_STAGES * STAGE_BYTES;
  static constexpr int RSTRIDE = BN + 4;                        // fp32 receive-row stride (16-byte rows, no bank conflicts)
  static constexpr int RECV_BYTES = KS * ROWS * RSTRIDE * 4;
  static constexpr int STG_STRIDE = 36;                         // staging row stride (32 columns + pad), floats
  static constexpr int STG_BYTES = HEAD_BM * STG_STRIDE * 4;    // one 32-column chunk of the accumulator
  static constexpr int BUF_BYTES = RECV_BYTES + STG_BYTES > RING_BYTES ? RECV_BYTES + STG_BYTES : RING_BYTES;
  static constexpr int SMEM_BYTES = 1024 + BUF_BYTES + 256;    // alignment slack, ring / receive, barriers
  static_assert(STAGE_BYTES % 1024 == 0 && HEAD_A_BYTES % 1024 == 0, "1024-byte aligned operand tiles");
  static_assert(BN % 32 == 0 && BN <= 256, "MMA N (and whole 32-column epilogue chunks)");
  static_assert(KS == 4 || KS == 8, "cluster size");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};

struct HeadArgs {
  int B, H, V;
  int kchunks;                 // K chunks of one CTA (H / (KS * HEAD_BK))
  uint16_t* logits;            // bf16 [B, ldl]
  int64_t ldl;
  int32_t* error_word;
};

// ---- tcgen05 / TMA / cluster primitives (PTX ISA 8.7, sm_100a) -------------

// Shared-memory matrix descriptor of a K-major operand tile whose rows are 128
// bytes (64 bf16) in the 128-byte swizzle: start address >> 4 in bits [0,14),
// leading byte offset (unused for this layout) 16 >> 4 in [16,30), stride byte
// offset 1024 >> 4 (one 8-row swizzle atom) in [32,46), version 1 in [46,48),
// layout type 2 (128-byte swizzle) in [61,64).  The tile starts on a 1024-byte
// boundary (base offset 0).
Q3S_DEV uint64_t head_smem_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(16 >> 4) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulator (bits [4,6) = 1), A and
// B bf16 (bits [7,10) = 1, [10,13) = 1), both K-major, N >> 3 in [17,23),
// M >> 4 in [24,29).
template <int BN>
__host__ __device__ constexpr uint32_t head_idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
         (static_cast<uint32_t>(HEAD_BM >> 4) << 24);
}

Q3S_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

Q3S_DEV void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrive on `bar` once every tcgen05.mma this thread issued before has completed.
Q3S_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

Q3S_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
Q3S_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
Q3S_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

Q3S_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

Q3S_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The shared::cluster address of `local_saddr` in CTA `rank` of the cluster.
Q3S_DEV uint32_t cluster_addr(uint32_t local_saddr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_saddr), "r"(rank));
  return remote;
}

Q3S_DEV void st_cluster_f4(uint32_t remote, float a0, float a1, float a2, float a3) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(remote), "f"(a0), "f"(a1), "f"(a2), "f"(a3)
               : "memory");
}

// Two fp32 values rounded to nearest-even bf16, `lo` in the low half.
Q3S_DEV uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// grid (V / BN, KS, ceil(B / HEAD_BM)), cluster (1, KS, 1)
template <int KS, int BN>
__global__ void __launch_bounds__(HEAD_NT, 1)
    head_gemm_kernel(const __grid_constant__ CUtensorMap tm_hidden, const __grid_constant__ CUtensorMap tm_weight,
                     const HeadArgs a) {
  using Tile = HeadTile<KS, BN>;
  constexpr int ROWS = Tile::ROWS;
  // the sampler launched after this grid as a programmatic dependent may
  // start its own preparation now; it waits for this grid before reading logits
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ __align__(1024) unsigned char head_smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(head_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Tile::BUF_BYTES);
  uint64_t* empty = full + HEAD_STAGES;
  uint64_t* done = empty + HEAD_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int t = static_cast<int>(threadIdx.x), w = t >> 5, lane = t & 31;
  const int n0 = static_cast<int>(blockIdx.x) * BN;
  const int m0 = static_cast<int>(blockIdx.z) * HEAD_BM;
  const int kc0 = static_cast<int>(blockIdx.y) * a.kchunks;  // this CTA's first K chunk
  const uint32_t rank = cluster_rank();

  if (t == 0) {
    for (int s = 0; s < HEAD_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *flag = 0;
    fence_mbar_init();
  }
  if (w == 0) {  // one warp allocates the accumulator's TMEM columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(Tile::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // ---- main loop: producer and MMA issuer --------------------------------
  if (t == 0) {
    for (int kc = 0; kc < a.kchunks; ++kc) {
      const int s = kc % HEAD_STAGES;
      if (kc >= HEAD_STAGES && !mbar_wait_bounded(&empty[s], ((kc / HEAD_STAGES) - 1) & 1)) {
        atomicOr(flag, 1);
        break;
      }
      unsigned char* st = smem + s * Tile::STAGE_BYTES;
      mbar_expect_tx(&full[s], Tile::STAGE_BYTES);
      const int kx = (kc0 + kc) * HEAD_BK;
      tma_load_2d(smem_u32(st), &tm_hidden, kx, m0, &full[s]);
      tma_load_2d(smem_u32(st + HEAD_A_BYTES), &tm_weight, kx, n0, &full[s]);
    }
  } else if (t == 32) {
    constexpr uint32_t idesc = head_idesc<BN>();
    for (int kc = 0; kc < a.kchunks; ++kc) {
      const int s = kc % HEAD_STAGES;
      if (!mbar_wait_bounded(&full[s], (kc / HEAD_STAGES) & 1)) {
        atomicOr(flag, 1);
        break;
      }
      tc_fence_after();
      const uint32_t sa = smem_u32(smem + s * Tile::STAGE_BYTES);
      const uint64_t da = head_smem_desc(sa), db = head_smem_desc(sa + HEAD_A_BYTES);
#pragma unroll
      for (int k = 0; k < HEAD_BK / 16; ++k)  // 16 bf16 = 32 bytes = 2 descriptor units per step
        umma_f16(tmem, da + 2 * k, db + 2 * k, idesc, (kc | k) != 0);
      umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
    }
    umma_commit(done);  // every MMA above has completed (none issued: arrives at once)
  }
  __syncwarp();
  const bool finished = mbar_wait_bounded(done, 0);
  if (!finished) atomicOr(flag, 1);
  tc_fence_after();
  tc_fence_before();
  // every CTA of the cluster is past its MMAs: all rings are free to receive
  cluster_sync();
  tc_fence_after();

  // ---- push: each accumulator row goes to the CTA that finishes it --------
  // row r of the tile (TMEM lane r) belongs to CTA r / 16 of the cluster; it
  // lands in that CTA's ring at receive slot `rank` (this CTA's K slice).  32
  // columns at a time: TMEM -> a padded local staging chunk (each lane one
  // row), then out with eight threads per 128-byte row segment, so every
  // warp's remote stores cover four contiguous row segments
  float* recv = reinterpret_cast<float*>(smem);
  float* stg = reinterpret_cast<float*>(smem + Tile::RECV_BYTES);
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    {
      float v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * w) << 16) + static_cast<uint32_t>(32 * c), v);
      float4* dst = reinterpret_cast<float4*>(stg + (32 * w + lane) * Tile::STG_STRIDE);
#pragma unroll
      for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < HEAD_BM * 8 / HEAD_NT; ++i) {
      const int f = t + HEAD_NT * i, row = f >> 3, q = f & 7;
      const float4 p = *reinterpret_cast<const float4*>(stg + row * Tile::STG_STRIDE + 4 * q);
      const uint32_t owner = static_cast<uint32_t>(row / ROWS);
      const uint32_t dst = cluster_addr(
          smem_u32(recv + (static_cast<int>(rank) * ROWS + row % ROWS) * Tile::RSTRIDE + 32 * c + 4 * q), owner);
      st_cluster_f4(dst, p.x, p.y, p.z, p.w);
    }
    __syncthreads();  // the staging chunk is reused
  }
  tc_fence_before();
  cluster_sync();  // every slice has arrived

  // ---- fixed-order sum of the KS K slices, rows [ROWS rank, ROWS (rank + 1)) --
  {
    constexpr int F4 = ROWS * BN / 4;  // float4s of the ROWS x BN slice
    for (int f = t; f < F4; f += HEAD_NT) {
      const int row = f / (BN / 4), c4 = f % (BN / 4);
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        const float4 p = *reinterpret_cast<const float4*>(recv + (k * ROWS + row) * Tile::RSTRIDE + 4 * c4);
        acc.x = __fadd_rn(acc.x, p.x);
        acc.y = __fadd_rn(acc.y, p.y);
        acc.z = __fadd_rn(acc.z, p.z);
        acc.w = __fadd_rn(acc.w, p.w);
      }
      const int grow = m0 + static_cast<int>(rank) * ROWS + row;
      if (grow < a.B)
        *reinterpret_cast<uint2*>(a.logits + static_cast<int64_t>(grow) * a.ldl + n0 + 4 * c4) =
            make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
    }
  }

  // ---- error path: wait (bounded) for this CTA's own copies and MMAs -------
  __syncthreads();
  if (*flag && t == 0) {
    if (!finished) (void)mbar_wait_bounded(done, 0);
    for (int s = 0; s < HEAD_STAGES && s < a.kchunks; ++s) (void)mbar_wait_bounded(&full[s], 0);
    if (a.error_word) atomicOr(a.error_word, Q3S_DEVERR_WAIT_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (w == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Tile::TMEM_COLS)
                 : "memory");
  }
}

}  // namespace q3s
