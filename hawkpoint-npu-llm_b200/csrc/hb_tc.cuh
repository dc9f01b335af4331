// hb_tc.cuh -- 5th-generation tensor-core (tcgen05) GEMM for batched rows.
//
// y[n][r] = sum_k W[r][k] * X[n][k] for a weight matrix W [rows x K] and up
// to 256 activation rows X [N x K], both BF16 in the packed row-group layout
// of runtime/layout.py: 8 rows x 16 bytes per core matrix, row group g at
// g * K * 16 bytes and chunk column j (8 K elements) at + j * 128.  That is
// the canonical no-swizzle K-major layout of a UMMA shared-memory operand,
// so one 1 KB bulk copy (cp.async.bulk, no tensor map, no multicast) moves
// 8 chunk columns of one row group straight into place.
//
// One CTA = one 128-row tile of W x one K slice (split-K when there are
// fewer tiles than SMs).  Warp 0 lane 0 streams the tile's A (16 row groups)
// and the B operand (N / 8 row groups) through an S-stage shared-memory ring,
// 64 K elements per stage; warp 1 lane 0 issues tcgen05.mma (M = 128, N =
// the padded batch, K = 16, BF16 -> FP32) into a TMEM accumulator and
// commits each stage back to the producer; all four warps then read the
// accumulator (warp w holds TMEM lanes 32w .. 32w + 31, one weight row per
// thread) and either finish the tile (one K slice) or leave an FP32 partial
// for the last slice to arrive, which sums the slices in slice order -- the
// result does not depend on which CTA finishes last.  Every wait is bounded
// (hb_device.cuh); on a timeout the kernel records it, still commits and
// drains what it issued, frees TMEM and returns.
#pragma once

#include "hb_device.cuh"

namespace hb {
namespace tc {

constexpr int kThreads = 128;
constexpr int kTileRows = 128;                 // MMA M
constexpr int kStageK = 64;                    // K elements per stage (8 chunk columns)
constexpr uint32_t kGroupStageBytes = 1024;    // one row group's 8 chunk columns
constexpr uint32_t kAStageBytes = 16 * kGroupStageBytes;
constexpr int kMaxN = 256;

// ---- tcgen05 PTX --------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (BF16 inputs, FP32 accumulate).
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `bar` when every tcgen05.mma this thread issued so far
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory operand descriptor, no swizzle, K-major: core matrices of
// 8 rows x 16 bytes; `lbo` = byte step between core matrices along K,
// `sbo` = byte step between 8-row groups (M / N); descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor, kind::f16: FP32 D, BF16 A and B, both K-major,
// M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(kTileRows >> 4) << 24);
}

__host__ __device__ inline int pad_n(int n) { return (n + 15) / 16 * 16; }
__host__ __device__ inline uint32_t tmem_cols(int npad) {
  uint32_t c = 32;
  while (c < static_cast<uint32_t>(npad)) c <<= 1;
  return c;
}

struct GemmParams {
  const uint8_t *w;   // packed weights, rows x K
  const uint8_t *x;   // packed activations, N (rounded up to 8) x K
  int rows, K, N;
  int npad;           // N rounded up to 16 (the MMA's N)
  int tiles, ksplit, kst;     // kst: K stages (K / 64) in all; slice s takes [s kst / ksplit, (s + 1) kst / ksplit)
  int stages;
  float *y;           // [N][rows] FP32 out
  float *ws;          // [tiles][ksplit][npad][128] FP32 partials (ksplit > 1)
  unsigned int *cnt;  // [tiles] slice arrivals (reset by the last)
  Ctrl *ctrl;
  uint64_t limit_ns;
};

__host__ __device__ inline size_t gemm_smem_bytes(int stages, int npad) {
  return static_cast<size_t>(stages) * (kAStageBytes + static_cast<size_t>(npad) * 128) + 16 * stages + 64;
}

// Bounded wait that does not raise on abort (cleanup paths).
__device__ __forceinline__ void mbar_wait_quiet(uint64_t *bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t start = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - start > limit_ns) return;
  }
}

__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ GemmParams P) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int S = P.stages;
  uint8_t *sa = smem;                                                   // [S][16 KB]
  uint8_t *sb = smem + static_cast<size_t>(S) * kAStageBytes;           // [S][npad * 128]
  uint64_t *full = reinterpret_cast<uint64_t *>(sb + static_cast<size_t>(S) * P.npad * 128);
  uint64_t *empty = full + S;
  uint64_t *done = empty + S;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  int *s_flag = reinterpret_cast<int *>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x / P.ksplit, split = blockIdx.x - tile * P.ksplit;
  const uint32_t ncols = tmem_cols(P.npad);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int groups_w = (P.rows + 7) / 8;
  const int groups_x = (P.N + 7) / 8;
  const int g0 = tile * 16;
  const int ga = min(16, groups_w - g0);  // row groups of this tile that exist
  const size_t rg_bytes = static_cast<size_t>(P.K) * 16;
  const int k0 = split * P.kst / P.ksplit;
  const int nk = (split + 1) * P.kst / P.ksplit - k0;  // K stages of this slice (>= 1)

  if (warp == 0 && lane == 0) {
    // producer
    const uint32_t bytes = static_cast<uint32_t>(ga + groups_x) * kGroupStageBytes;
    int issued = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      const uint32_t ph = static_cast<uint32_t>(i / S) & 1u;
      if (i >= S && !mbar_wait(&empty[s], ph ^ 1u, P.ctrl, P.limit_ns, kWhereEmpty)) break;
      mbar_arrive_expect_tx(&full[s], bytes);
      const size_t koff = static_cast<size_t>(k0 + i) * kGroupStageBytes;
      for (int g = 0; g < ga; ++g)
        bulk_g2s(sa + static_cast<size_t>(s) * kAStageBytes + g * kGroupStageBytes,
                 P.w + static_cast<size_t>(g0 + g) * rg_bytes + koff, kGroupStageBytes, &full[s]);
      for (int b = 0; b < groups_x; ++b)
        bulk_g2s(sb + static_cast<size_t>(s) * P.npad * 128 + b * kGroupStageBytes,
                 P.x + static_cast<size_t>(b) * rg_bytes + koff, kGroupStageBytes, &full[s]);
      ++issued;
    }
    // every copy this thread issued has landed before the CTA can exit
    for (int i = max(0, issued - S); i < issued; ++i)
      mbar_wait_quiet(&full[i % S], static_cast<uint32_t>(i / S) & 1u, P.limit_ns);
  } else if (warp == 1 && lane == 0) {
    // MMA issuer
    const uint32_t idesc = idesc_bf16(P.npad);
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      const uint32_t ph = static_cast<uint32_t>(i / S) & 1u;
      if (!mbar_wait(&full[s], ph, P.ctrl, P.limit_ns, kWhereFull)) break;
      tc_fence_after();
      const uint32_t a = smem_u32(sa + static_cast<size_t>(s) * kAStageBytes);
      const uint32_t b = smem_u32(sb + static_cast<size_t>(s) * P.npad * 128);
#pragma unroll
      for (int kk = 0; kk < kStageK / 16; ++kk) {
        umma_bf16(tmem, smem_desc(a + kk * 256, 128, kGroupStageBytes), smem_desc(b + kk * 256, 128, kGroupStageBytes),
                  idesc, (i | kk) != 0 ? 1u : 0u);
      }
      umma_commit(&empty[s]);  // the slot is free once these MMAs have read it
    }
    umma_commit(done);  // also on an early exit: nothing in flight when TMEM is freed
  }
  __syncwarp();
  // epilogue: wait for the accumulator (or, after an abort, for the MMAs in flight)
  const bool ok = __syncthreads_and(mbar_wait(done, 0, P.ctrl, P.limit_ns, kWhereFull) &&
                                    ld_volatile_int(&P.ctrl->abort) == 0) != 0;
  tc_fence_after();
  const int row = g0 * 8 + warp * 32 + lane;  // this thread's weight row
  const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  if (ok) {
    float *part = P.ksplit > 1 ? P.ws + (static_cast<size_t>(tile) * P.ksplit + split) * P.npad * kTileRows : nullptr;
    for (int c0 = 0; c0 < P.npad; c0 += 16) {
      uint32_t v[16];
      tmem_ld16(taddr + c0, v);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = c0 + j;
        if (part != nullptr) {
          part[static_cast<size_t>(n) * kTileRows + warp * 32 + lane] = __uint_as_float(v[j]);
        } else if (n < P.N && row < P.rows) {
          P.y[static_cast<size_t>(n) * P.rows + row] = __uint_as_float(v[j]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ncols);
  if (!ok || P.ksplit == 1) return;
  // split-K: the last slice to arrive sums the slices in order
  if (threadIdx.x == 0) {
    __threadfence();
    *s_flag = atomicAdd(&P.cnt[tile], 1u) == static_cast<unsigned>(P.ksplit - 1) ? 1 : 0;
  }
  __syncthreads();
  if (*s_flag == 0) return;
  __threadfence();
  if (threadIdx.x == 0) P.cnt[tile] = 0u;
  const float *base = P.ws + static_cast<size_t>(tile) * P.ksplit * P.npad * kTileRows;
  if (row < P.rows) {
    for (int n = 0; n < P.N; ++n) {
      float acc = 0.f;
      for (int s2 = 0; s2 < P.ksplit; ++s2)
        acc += __ldcg(base + (static_cast<size_t>(s2) * P.npad + n) * kTileRows + warp * 32 + lane);
      P.y[static_cast<size_t>(n) * P.rows + row] = acc;
    }
  }
}

}  // namespace tc
}  // namespace hb
