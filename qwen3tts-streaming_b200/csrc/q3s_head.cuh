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
// each CTA finishing 128 / KS of the 128 rows.  For V = 3072: KS = 4, BN = 96,
// 32 x 4 = 128 CTAs per 128 rows, 224 KB of operands each.
//
// Per CTA (128 threads):
//   warp 0 lane 0   TMA producer: 2-D tiled loads (cp.async.bulk.tensor, no
//                   multicast) of the hidden tile [128 x 64] and the weight
//                   tile [BN x 64] per K chunk into a ring of as many stages
//                   as shared memory holds (5-8: most of a CTA's operands are
//                   in flight at once), 128-byte swizzled (the layout the MMA
//                   descriptors below name);
//   warp 1 lane 0   MMA issuer: tcgen05.mma.cta_group::1.kind::f16 (bf16 x
//                   bf16 -> fp32), M = 128, N = BN, K = 16 per instruction,
//                   accumulator in TMEM; tcgen05.commit frees a stage and
//                   finally signals the epilogue;
//   each warp       epilogue, independently: tcgen05.ld of its 32 TMEM lanes
//                   (rows) into a staging copy of the partial tile in the
//                   now idle ring, then one bulk copy per owning CTA
//                   (cp.async.bulk shared::cta -> shared::cluster, completing
//                   on the owner's receive mbarrier) of the rows that CTA
//                   finishes;
//   all threads     wait for the KS - 1 incoming slices on the receive
//                   mbarrier, then the fixed-order sum of the KS slices
//                   (slice k from CTA k; this CTA's own from its staging),
//                   rounded to bf16.
// No cluster-wide barrier sits on the critical path: one after the barrier
// initialisation (a remote mbarrier must be initialised before a copy
// completes on it; every CTA has long passed it when its copies go out) and
// one before exit (every copy into every CTA of the cluster has landed, so no
// CTA leaves while a copy still reads its staging), split around the sum.
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
constexpr int HEAD_MAX_STAGES = 8;
constexpr int HEAD_NT = 128;
constexpr int HEAD_A_BYTES = HEAD_BM * HEAD_BK * 2;   // 16 KB
constexpr int HEAD_BAR_BYTES = 256;
constexpr int HEAD_SMEM_LIMIT = 227 * 1024;     // per CTA
// Preferred budget: leaves an SM room for one CTA of the row sampler launched
// behind the head as a programmatic dependent (~27 KB of shared memory and
// 384 threads at V = 3072), which then runs its preparation while the head
// still computes and starts on the logits the moment the head's grid is done.
constexpr int HEAD_SMEM_SHARED = 192 * 1024;

// One configuration: KS CTAs per cluster (one K slice each, 4 or 8) and a
// vocabulary tile of BN entries (the MMA's N).
template <int KS, int BN>
struct HeadTile {
  static constexpr int ROWS = HEAD_BM / KS;                     // rows each CTA of a cluster finishes
  static constexpr int TMEM_COLS = BN <= 128 ? 128 : 256;       // power of two >= BN
  static constexpr int B_BYTES = BN * HEAD_BK * 2;
  static constexpr int STAGE_BYTES = HEAD_A_BYTES + B_BYTES;   // multiple of 1024
  static constexpr int SLOT_BYTES = ROWS * BN * 4;              // one K slice of the rows a CTA finishes
  static constexpr int RECV_BYTES = (KS - 1) * SLOT_BYTES;      // the other CTAs' slices
  static constexpr int STAGING_BYTES = HEAD_BM * BN * 4;        // this CTA's whole partial tile (in the ring)
  static constexpr int fit(int limit) { return (limit - 1024 - HEAD_BAR_BYTES - RECV_BYTES) / STAGE_BYTES; }
  // the shared budget when it still holds 3 stages and the staging copy
  static constexpr bool SHARED_OK = fit(HEAD_SMEM_SHARED) >= 3 && fit(HEAD_SMEM_SHARED) * STAGE_BYTES >= STAGING_BYTES;
  static constexpr int FIT = fit(SHARED_OK ? HEAD_SMEM_SHARED : HEAD_SMEM_LIMIT);
  static constexpr int STAGES = FIT < HEAD_MAX_STAGES ? FIT : HEAD_MAX_STAGES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int SMEM_BYTES = 1024 + RING_BYTES + RECV_BYTES + HEAD_BAR_BYTES;  // + alignment slack
  static_assert(STAGE_BYTES % 1024 == 0 && HEAD_A_BYTES % 1024 == 0, "1024-byte aligned operand tiles");
  static_assert(BN % 32 == 0 && BN <= 256, "MMA N (and whole 32-column epilogue chunks)");
  static_assert(KS == 4 || KS == 8, "cluster size");
  static_assert(STAGES >= 2 && STAGING_BYTES <= RING_BYTES, "ring");
  static_assert(SLOT_BYTES % 16 == 0, "bulk copy sizes");
  static_assert(SMEM_BYTES <= HEAD_SMEM_LIMIT, "shared memory");
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

// The cluster barrier in two halves: every thread of every CTA arrives, and
// wait returns once all have.
Q3S_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Arrival that orders no memory: for barriers that only say "this CTA got
// this far" (the mbarrier initialisation before it is released by its own
// fence, and a copy's completion is observed on the receiving mbarrier).
Q3S_DEV void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }

// The shared::cluster address of `local_saddr` in CTA `rank` of the cluster.
Q3S_DEV uint32_t cluster_addr(uint32_t local_saddr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_saddr), "r"(rank));
  return remote;
}

// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned)
// from this CTA's shared memory to shared::cluster address `dst` (another CTA
// of the cluster), completing `bytes` of transactions on the mbarrier at
// shared::cluster address `bar` (in the destination CTA).
Q3S_DEV void bulk_s2cluster(uint32_t dst, uint32_t src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "r"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Generic-proxy shared-memory writes of this thread, ordered before later
// async-proxy reads of them (the bulk copies above).
Q3S_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Two fp32 values rounded to nearest-even bf16, `lo` in the low half.
Q3S_DEV uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Receive slot, in CTA `owner`, of the slice sent by CTA `sender` (!= owner).
Q3S_DEV int head_slot(int sender, int owner) { return sender < owner ? sender : sender - 1; }

// grid (V / BN, KS, ceil(B / HEAD_BM)), cluster (1, KS, 1)
template <int KS, int BN>
__global__ void __launch_bounds__(HEAD_NT, 1)
    head_gemm_kernel(const __grid_constant__ CUtensorMap tm_hidden, const __grid_constant__ CUtensorMap tm_weight,
                     const HeadArgs a) {
  using Tile = HeadTile<KS, BN>;
  constexpr int ROWS = Tile::ROWS;
  constexpr int STAGES = Tile::STAGES;
  constexpr int F4_ROW = BN / 4;  // float4s per partial-tile row
  // the sampler launched after this grid as a programmatic dependent may
  // start its own preparation now; it waits for this grid before reading logits
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ __align__(1024) unsigned char head_smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(head_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* recv = reinterpret_cast<float*>(smem + Tile::RING_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Tile::RING_BYTES + Tile::RECV_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint64_t* recv_bar = done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  int* flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int t = static_cast<int>(threadIdx.x), w = t >> 5, lane = t & 31;
  const int n0 = static_cast<int>(blockIdx.x) * BN;
  const int m0 = static_cast<int>(blockIdx.z) * HEAD_BM;
  const int kc0 = static_cast<int>(blockIdx.y) * a.kchunks;  // this CTA's first K chunk
  const int rank = static_cast<int>(cluster_rank());

  auto load_chunk = [&](int kc) {
    const int s = kc % STAGES;
    unsigned char* st = smem + s * Tile::STAGE_BYTES;
    mbar_expect_tx(&full[s], Tile::STAGE_BYTES);
    const int kx = (kc0 + kc) * HEAD_BK;
    tma_load_2d(smem_u32(st), &tm_hidden, kx, m0, &full[s]);
    tma_load_2d(smem_u32(st + HEAD_A_BYTES), &tm_weight, kx, n0, &full[s]);
  };
  const int first = a.kchunks < STAGES ? a.kchunks : STAGES;  // chunks whose stage starts empty
  if (t == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_init(recv_bar, 1);
    mbar_expect_tx(recv_bar, (KS - 1) * Tile::SLOT_BYTES);  // the only arrival; the copies complete the bytes
    *flag = 0;
    fence_mbar_init();
    // the first loads fly while warp 1 allocates the accumulator
    for (int kc = 0; kc < first; ++kc) load_chunk(kc);
  }
  if (w == 1) {  // the MMA warp allocates the accumulator's TMEM columns (and frees them)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(Tile::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cluster_arrive_relaxed();  // this CTA's receive mbarrier is initialised (fenced above; waited on before the first copy)
  const uint32_t tmem = *tmem_slot;

  // ---- main loop: producer and MMA issuer --------------------------------
  if (t == 0) {
    for (int kc = first; kc < a.kchunks; ++kc) {
      const int s = kc % STAGES;
      if (!mbar_wait_bounded(&empty[s], ((kc / STAGES) - 1) & 1)) {
        atomicOr(flag, 1);
        break;
      }
      load_chunk(kc);
    }
  } else if (t == 32) {
    constexpr uint32_t idesc = head_idesc<BN>();
    for (int kc = 0; kc < a.kchunks; ++kc) {
      const int s = kc % STAGES;
      if (!mbar_wait_bounded(&full[s], (kc / STAGES) & 1)) {
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

  // ---- stage and send: each warp on its own ------------------------------
  // warp w holds TMEM lanes (tile rows) [32 w, 32 w + 32) and writes them into
  // the staging copy of the partial tile (row-major, BN floats a row) that
  // now occupies the idle ring; float4 column q of row r sits at q ^ (r & 7),
  // so the eight rows of a quarter-warp's 16-byte stores hit eight different
  // bank groups.  Rows [ROWS d, ROWS (d + 1)) then go to CTA d in one copy.
  float* stg = reinterpret_cast<float*>(smem);
  {
    const int row = 32 * w + lane;
    float4* rowp = reinterpret_cast<float4*>(stg + row * BN);
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * w) << 16) + static_cast<uint32_t>(32 * c), v);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        rowp[(8 * c + q) ^ (row & 7)] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  // every TMEM read is done: the accumulator can go now, unless a wait timed
  // out (an MMA may still be running: then it goes last).  Every thread that
  // set the flag so far sees its own write, so `clean` is one value per CTA.
  const bool clean = __syncthreads_and(*flag == 0) != 0;
  if (w == 1 && clean) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Tile::TMEM_COLS)
                 : "memory");
  }
  cluster_wait();  // every CTA's receive mbarrier is initialised
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < 32 / ROWS; ++h) {  // the owners of this warp's rows
      const int owner = (32 * w) / ROWS + h;
      if (owner == rank) continue;
      const uint32_t dst = cluster_addr(
          smem_u32(recv) + static_cast<uint32_t>(head_slot(rank, owner) * Tile::SLOT_BYTES), owner);
      bulk_s2cluster(dst, smem_u32(stg + owner * ROWS * BN), Tile::SLOT_BYTES,
                     cluster_addr(smem_u32(recv_bar), owner));
    }
  }

  // ---- fixed-order sum of the KS K slices, rows [ROWS rank, ROWS (rank + 1)) --
  bool received = true;
  if (t == 0 && !mbar_wait_bounded(recv_bar, 0)) {
    received = false;
    atomicOr(flag, 1);
  }
  __syncthreads();  // the slices are in, and this CTA's own staging rows are written
  cluster_arrive_relaxed();  // every copy into this CTA has landed (observed on recv_bar)
  {
    constexpr int PER = ROWS * F4_ROW / HEAD_NT;  // float4s of the slice per thread
    static_assert(ROWS * F4_ROW % HEAD_NT == 0, "whole float4s per thread");
    const float4* own = reinterpret_cast<const float4*>(stg) + rank * ROWS * F4_ROW;
    const float4* in = reinterpret_cast<const float4*>(recv);
    float4 acc[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) acc[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < KS; ++k) {  // fixed order: K slice 0 first
      const float4* src = k == rank ? own : in + head_slot(k, rank) * ROWS * F4_ROW;
      float4 p[PER];
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int f = t + HEAD_NT * i, row = f / F4_ROW, c4 = f % F4_ROW;
        p[i] = src[row * F4_ROW + (c4 ^ (row & 7))];  // ROWS is a multiple of 8: row & 7 is the tile row's
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        acc[i].x = __fadd_rn(acc[i].x, p[i].x);
        acc[i].y = __fadd_rn(acc[i].y, p[i].y);
        acc[i].z = __fadd_rn(acc[i].z, p[i].z);
        acc[i].w = __fadd_rn(acc[i].w, p[i].w);
      }
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int f = t + HEAD_NT * i, row = f / F4_ROW, c4 = f % F4_ROW;
      const int grow = m0 + rank * ROWS + row;
      if (grow < a.B)
        *reinterpret_cast<uint2*>(a.logits + static_cast<int64_t>(grow) * a.ldl + n0 + 4 * c4) =
            make_uint2(pack_bf16x2(acc[i].x, acc[i].y), pack_bf16x2(acc[i].z, acc[i].w));
    }
  }
  cluster_wait();  // every copy in the cluster has landed: the staging may go

  // ---- error path: wait (bounded) for this CTA's own copies and MMAs -------
  if (*flag && t == 0) {
    if (!finished) (void)mbar_wait_bounded(done, 0);
    if (!received) (void)mbar_wait_bounded(recv_bar, 0);
    for (int s = 0; s < STAGES && s < a.kchunks; ++s) (void)mbar_wait_bounded(&full[s], 0);
    if (a.error_word) atomicOr(a.error_word, Q3S_DEVERR_WAIT_TIMEOUT);
  }
  if (!clean) {
    tc_fence_before();
    __syncthreads();
    if (w == 1) {
      tc_fence_after();
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Tile::TMEM_COLS)
                   : "memory");
    }
  }
}

}  // namespace q3s
