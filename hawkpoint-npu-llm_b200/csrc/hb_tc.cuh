// hb_tc.cuh -- 5th-generation tensor-core (tcgen05) GEMM for batched rows.
//
// y[n][r] = sum_k W[r][k] * X[n][k] for a weight matrix W [rows x K] and up
// to 256 activation rows X [N x K], both BF16 in the packed row-group layout
// of runtime/layout.py: 8 rows x 16 bytes per core matrix, row group g at
// g * K * 16 bytes and chunk column j (8 K elements) at + j * 128.  That is
// the canonical no-swizzle K-major layout of a UMMA shared-memory operand:
// one stage (64 K elements) of a row group is 1 KB, contiguous, and a stage
// of several row groups lands in shared memory already in MMA order.  Each
// operand is addressed through a 3-D tensor map over that layout (1 KB
// stage piece x K stage x row group), so one TMA load (no multicast) fetches
// a whole stage of a tile: per-copy cost, not bytes, limits an SM that
// streams 1 KB pieces one bulk copy each (about 25 GB/s per SM against
// about 80 GB/s for one load per stage, measured on B200).  Row groups past
// the end of W or of the batch read as zeros.
//
// One CTA = one 128-row tile of W x one K slice (split-K when there are
// fewer tiles than SMs).  Warp 0 lane 0 streams the tile's A (16 row groups)
// and the B operand (npad / 8 row groups) through an S-stage shared-memory
// ring, 64 K elements per stage; warp 1 lane 0 issues tcgen05.mma (M = 128, N =
// the padded batch, K = 16, BF16 -> FP32) into a TMEM accumulator and
// commits each stage back to the producer; all four warps then read the
// accumulator (warp w holds TMEM lanes 32w .. 32w + 31, one weight row per
// thread) into shared memory.  One K slice finishes the tile there; the K
// slices of a tile run as one thread-block cluster and sum their partials
// through distributed shared memory in slice order, each slice finishing a
// share of the columns (the result does not depend on the order the slices
// finish in).  Every mbarrier wait is bounded (hb_device.cuh); on a timeout
// the kernel records it, still commits and drains what it issued, frees
// TMEM, passes the cluster barriers (which every CTA reaches) and returns.
#pragma once

#include <cuda.h>

#include "hb_attn.cuh"

namespace hb {
namespace tc {

constexpr int kThreads = 128;
constexpr int kTileRows = 128;                 // MMA M
constexpr int kStageK = 64;                    // K elements per stage (8 chunk columns)
constexpr uint32_t kGroupStageBytes = 1024;    // one row group's 8 chunk columns
constexpr uint32_t kAStageBytes = 16 * kGroupStageBytes;
constexpr int kMaxN = 256;
constexpr int kHeadDimTc = 64;

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

// One box of a 3-D tensor map (coordinates x, y, z) into shared memory,
// completion on `bar`.  No multicast.
__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *map, int x, int y, int z,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(smem_u32(smem_dst)), "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

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

// Row metadata of a batched step (device arrays of n entries).
struct Rows {
  const int *slot, *pos, *tok;
};

struct KvArgs {
  const __nv_bfloat16 *qkv;  // [N][QKV] BF16 (biased q / k / v)
  int QKV, QH, KVH, group, H;
  const float *cos, *sin;    // [ctx][32]
  __nv_bfloat16 *kv;         // [slots][L][KVH][K | V][ctx][64], swizzled rows
  int L, layer, ctx;
};

__device__ __forceinline__ uint8_t *kv_rows(const KvArgs &A, int slot, int j, int kind) {
  return reinterpret_cast<uint8_t *>(A.kv) +
         ((((static_cast<size_t>(slot) * A.L + A.layer) * A.KVH + j) * 2 + kind) * A.ctx * kHeadDimTc) * 2;
}

struct GemmParams {
  // packed weights (rows x K) and activations (N x K) as 3-D maps of 32-bit
  // words: {256 (one 1 KB stage piece), K / 64 stages, row groups}, boxes
  // {256, 1, 16} and {256, 1, npad / 8}
  CUtensorMap map_w, map_x;
  int rows, K, N;
  int npad;           // N rounded up to 16 (the MMA's N)
  int tiles, ksplit, kst;     // kst: K stages (K / 64) in all; slice s takes [s kst / ksplit, (s + 1) kst / ksplit)
  int stages;
  float *y;           // kEpiF32: [N][rows] FP32 out; kEpiLogits: optional FP32 logits [N][rows]
  const float *bias;  // kEpiQkv: [rows] FP32 (nullptr: none)
  const __nv_bfloat16 *resid;  // kEpiResid: [N][rows] BF16
  __nv_bfloat16 *out;  // kEpiQkv (q rows) / kEpiResid: [N][rows] BF16; kEpiSwiglu: packed [N][rows / 2]
  KvArgs kv;           // kEpiQkv: the K / V cache the k and v rows go to
  Rows R;              // kEpiQkv: each column's slot and position
  float *part_val;    // kEpiLogits: [tiles][pstride] per-tile maxima
  int *part_idx;
  int pstride;
  Ctrl *ctrl;
  uint64_t limit_ns;
};

// Shared memory of a GEMM CTA: the operand ring, reused after the last MMA
// for the epilogue -- the tile's FP32 results (this slice's partial)
// [npad][128] and, with K slices, the slice's summed share of columns --
// then the barriers.
__host__ __device__ inline int gemm_share(int npad, int ksplit) { return (npad + ksplit - 1) / ksplit; }
__host__ __device__ inline size_t gemm_epi_bytes(int npad, int ksplit) {
  return (static_cast<size_t>(npad) + (ksplit > 1 ? gemm_share(npad, ksplit) : 0)) * kTileRows * 4;
}
__host__ __device__ inline size_t gemm_data_bytes(int stages, int npad, int ksplit) {
  const size_t ring = static_cast<size_t>(stages) * (kAStageBytes + static_cast<size_t>(npad) * 128);
  const size_t epi = gemm_epi_bytes(npad, ksplit);
  return ((ring > epi ? ring : epi) + 1023) / 1024 * 1024;
}
__host__ __device__ inline size_t gemm_smem_bytes(int stages, int npad, int ksplit) {
  return gemm_data_bytes(stages, npad, ksplit) + 16 * stages + 64;
}

// ---- programmatic dependent launch ----------------------------------------------
// Lets the next kernel of the stream be scheduled now (its CTAs start on free
// SMs and may prefetch weights); no-op without the launch attribute.
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Waits until the kernels this one depends on have completed and their
// writes are visible; no-op without the launch attribute.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- thread-block cluster (the K slices of one tile) ---------------------------
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// The address of the same shared-memory variable in cluster CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_cluster_f32x4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
constexpr int kMaxSlices = 8;  // portable cluster size

// What a GEMM does with y[n][r] (cpu_backend.py rounding points):
enum : int {
  kEpiF32 = 0,     // y -> FP32 [N][rows]
  kEpiQkv = 1,     // bf16(bf16(y) + bias[r]): q rows -> BF16 [N][rows]; k rows rotated and v rows
                   // appended to the K / V cache at the column's slot / position (qkv, :78-93, :134-143)
  kEpiResid = 2,   // bf16(bf16(y) + resid[n][r]) -> BF16 [N][rows]      (o / down, :145-151, :166-171)
  kEpiSwiglu = 3,  // rows are gate / up row-group pairs: bf16(silu(bf16 g) * bf16 u) -> packed act (:154-165)
  kEpiLogits = 4,  // FP32 logits (optional) and each row's maximum over the tile (np.argmax order)
};

// Bounded wait that does not raise on abort (cleanup paths).
__device__ __forceinline__ void mbar_wait_quiet(uint64_t *bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t start = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - start > limit_ns) return;
  }
}

// Row n of `out` (packed row-group layout) = bf16((x * inv_rms) * gamma) of
// the BF16 row x (cpu_backend.py:71-76); one warp, lane l taking 16-byte
// chunks l, l + 32, ... (held in registers for rows of up to 1024 values).
// Reads through L2, so rows that other CTAs of the same kernel wrote are
// seen.
__device__ __forceinline__ float sum_squares8(const uint4 &w, float ss) {
  const uint32_t in[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    ss = fmaf(bf_lo(in[e]), bf_lo(in[e]), ss);
    ss = fmaf(bf_hi(in[e]), bf_hi(in[e]), ss);
  }
  return ss;
}

// Chunk c (8 values, gamma g) of a normalised row into the packed layout.
__device__ __forceinline__ void put_norm8(const uint4 &w, const float (&g)[8], float inv, int c, int kc, uint8_t *out,
                                          int n) {
  const uint32_t in[4] = {w.x, w.y, w.z, w.w};
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float a = __fmul_rn(__fmul_rn(bf_lo(in[e]), inv), g[2 * e]);
    const float b = __fmul_rn(__fmul_rn(bf_hi(in[e]), inv), g[2 * e + 1]);
    o[e] = pack_bf16x2(a, b);
  }
  *reinterpret_cast<uint4 *>(out + (static_cast<size_t>(n >> 3) * kc + c) * 128 + (n & 7) * 16) =
      make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ void load_gamma8(const float *gamma, int c, float (&g)[8]) {
  const float4 g0 = __ldg(reinterpret_cast<const float4 *>(gamma) + 2 * c);
  const float4 g1 = __ldg(reinterpret_cast<const float4 *>(gamma) + 2 * c + 1);
  g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w;
  g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
}

// Rows n[i] of `out` (packed row-group layout) = bf16((x * inv_rms) * gamma)
// of the BF16 rows x[i] (cpu_backend.py:71-76) for the R rows with n[i] >= 0;
// one warp, lane l taking 16-byte chunks l, l + 32, ... of every row.  Every
// load (both rows, gamma) is issued before the first store, and rows of up
// to 1024 values stay in registers.  Reads through L2, so rows that other
// CTAs of the same kernel wrote are seen.
template <int R>
__device__ __forceinline__ void norm_pack_rows(const __nv_bfloat16 *const (&x)[R], const int (&n)[R],
                                               const float *gamma, float eps, int H, uint8_t *out) {
  constexpr int kHeld = 4;
  const int lane = threadIdx.x & 31, kc = H / 8;
  uint4 held[R][kHeld];
  float g[kHeld][8];
#pragma unroll
  for (int i = 0; i < kHeld; ++i) {
    const int c = lane + 32 * i;
#pragma unroll
    for (int r = 0; r < R; ++r)
      held[r][i] = n[r] >= 0 && c < kc ? __ldcg(reinterpret_cast<const uint4 *>(x[r]) + c) : make_uint4(0, 0, 0, 0);
    if (c < kc) load_gamma8(gamma, c, g[i]);
  }
  float inv[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kHeld; ++i)
      if (lane + 32 * i < kc) ss = sum_squares8(held[r][i], ss);
    if (n[r] >= 0)
      for (int c = lane + 32 * kHeld; c < kc; c += 32) ss = sum_squares8(__ldcg(reinterpret_cast<const uint4 *>(x[r]) + c), ss);
    const float total = warp_sum(ss);
    inv[r] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(H)), eps)));
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (n[r] < 0) continue;
#pragma unroll
    for (int i = 0; i < kHeld; ++i)
      if (lane + 32 * i < kc) put_norm8(held[r][i], g[i], inv[r], lane + 32 * i, kc, out, n[r]);
    for (int c = lane + 32 * kHeld; c < kc; c += 32) {
      float gg[8];
      load_gamma8(gamma, c, gg);
      put_norm8(__ldcg(reinterpret_cast<const uint4 *>(x[r]) + c), gg, inv[r], c, kc, out, n[r]);
    }
  }
}

__device__ __forceinline__ void norm_pack_row(const __nv_bfloat16 *x, const float *gamma, float eps, int H,
                                              uint8_t *out, int n) {
  const __nv_bfloat16 *const xs[1] = {x};
  const int ns[1] = {n};
  norm_pack_rows<1>(xs, ns, gamma, eps, H, out);
}

// Residual columns a kEpiResid CTA stages in shared memory while its MMAs
// run (the first kResPre of the columns it finishes; the rest are read in
// the epilogue).
constexpr int kResPre = 40;

// Epilogue inputs a GEMM CTA stages in shared memory before its epilogue,
// for the columns n0 + c it finishes:
// kEpiResid: res[c * 128 + row in tile], the residual (c < kResPre);
// kEpiQkv (tiles with k / v rows): pos[c], slot[c] (every c), and cs[c * 64 +
// d] = cos, cs[c * 64 + 32 + d] = sin of the column's position (c < kResPre).
struct EpiSmem {
  const __nv_bfloat16 *res;
  const int *pos, *slot;
  const float *cs;
};

// The epilogue of columns [n0, n1) of a tile from its FP32 results in
// shared memory (stage[(n - n0) * 128 + row in tile]); 128 threads.
template <int EPI>
__device__ __forceinline__ void finish_tile(const GemmParams &P, float *stage, int tile, int n0, int n1,
                                            const EpiSmem &E) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = tile * kTileRows;
  // with 128 threads stepping by 128, a thread's row within the tile is
  // fixed: threadIdx.x; its columns are n0 + k
  const int row = row0 + threadIdx.x;
  const bool row_ok = row < P.rows;
  if constexpr (EPI == kEpiF32 || EPI == kEpiResid) {
    if (!row_ok) return;
    // the residual reads of kBatch columns are all in flight before the
    // first store (one memory round per kBatch columns, not per column)
    constexpr int kBatch = 8;
    for (int c0 = n0; c0 < n1; c0 += kBatch) {
      float r[kBatch];
      if constexpr (EPI == kEpiResid) {
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int c = c0 + u - n0;
          r[u] = c0 + u >= n1     ? 0.f
                 : c < kResPre ? bf2f(E.res[c * kTileRows + threadIdx.x])
                               : bf2f(P.resid[static_cast<size_t>(c0 + u) * P.rows + row]);
        }
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        if (c0 + u >= n1) break;
        const float v = stage[(c0 + u - n0) * kTileRows + threadIdx.x];
        const size_t o = static_cast<size_t>(c0 + u) * P.rows + row;
        if constexpr (EPI == kEpiF32) {
          P.y[o] = v;
        } else {
          P.out[o] = f2bf(__fadd_rn(rbf(v), r[u]));
        }
      }
    }
  } else if constexpr (EPI == kEpiQkv) {
    // BF16 biased values back into the stage; q rows to out
    const int qrows = P.kv.QH * kHeadDimTc;
    if (row_ok) {
      const float bias = P.bias != nullptr ? P.bias[row] : 0.f;
      for (int n = n0; n < n1; ++n) {
        const int idx = (n - n0) * kTileRows + threadIdx.x;
        float yv = rbf(stage[idx]);
        if (P.bias != nullptr) yv = __fadd_rn(yv, bias);
        const __nv_bfloat16 b = f2bf(yv);
        stage[idx] = bf2f(b);
        if (row < qrows) P.out[static_cast<size_t>(n) * P.rows + row] = b;
      }
    }
    // the tile's two heads per column: a k head is rotated at the column's
    // position and stored as K, a v head stored as V (one warp per head)
    if (row0 + kTileRows <= P.kv.QH * kHeadDimTc) return;  // q rows only
    __syncthreads();  // the stage is read across threads next
    // kBatch units per warp per pass, their RoPE table reads in flight together
    constexpr int kBatch = 4, kWarps = kThreads / 32;
    const int units = (n1 - n0) * 2;
    for (int u0 = warp; u0 < units; u0 += kBatch * kWarps) {
      float cs[kBatch], sn[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int u = u0 + j * kWarps;
        const int head = row0 / kHeadDimTc + (u & 1);
        cs[j] = sn[j] = 0.f;
        if (u < units && head >= P.kv.QH && head < P.kv.QH + P.kv.KVH) {
          const int c = u >> 1;
          if (c < kResPre) {
            cs[j] = E.cs[c * 64 + lane];
            sn[j] = E.cs[c * 64 + 32 + lane];
          } else {
            const int p = E.pos[c];
            cs[j] = P.kv.cos[p * 32 + lane];
            sn[j] = P.kv.sin[p * 32 + lane];
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int u = u0 + j * kWarps;
        if (u >= units) break;
        const int n = n0 + (u >> 1), hh = u & 1;
        const int head = row0 / kHeadDimTc + hh;
        if (head < P.kv.QH || head * kHeadDimTc >= P.rows) continue;
        const float *v = stage + (n - n0) * kTileRows + hh * kHeadDimTc;
        const int p = E.pos[n - n0], slot = E.slot[n - n0];
        if (head < P.kv.QH + P.kv.KVH) {
          __nv_bfloat16 lo, hi;
          rope_vals(v[lane], v[lane + 32], cs[j], sn[j], lo, hi);
          put_k(kv_rows(P.kv, slot, head - P.kv.QH, 0), p, lane, lo, hi);
        } else {
          put_v(kv_rows(P.kv, slot, head - P.kv.QH - P.kv.KVH, 1), p, lane,
                pack_bf16x2(v[2 * lane], v[2 * lane + 1]));
        }
      }
    }
  } else if constexpr (EPI == kEpiSwiglu) {
    // pair q of the tile: gate rows q*16 + rr, up rows q*16 + 8 + rr, act
    // column (row0 / 16 + q) * 8 + rr; 8 outputs = one 16-byte chunk
    const int inter = P.rows / 2, kc = inter / 8;
    for (int idx = threadIdx.x; idx < (n1 - n0) * 8; idx += kThreads) {
      const int n = n0 + (idx >> 3), q = idx & 7;
      if (row0 + q * 16 >= P.rows) continue;
      uint32_t w4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float a[2];
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int rr = 2 * e + h2;
          const float g = rbf(stage[(n - n0) * kTileRows + q * 16 + rr]);
          const float u = rbf(stage[(n - n0) * kTileRows + q * 16 + 8 + rr]);
          const float ex = expf(-fminf(fmaxf(g, -80.f), 80.f));
          a[h2] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, ex)), u);
        }
        w4[e] = pack_bf16x2(a[0], a[1]);
      }
      uint8_t *dst = reinterpret_cast<uint8_t *>(P.out) +
                     (static_cast<size_t>(n >> 3) * kc + (row0 / 16 + q)) * 128 + (n & 7) * 16;
      *reinterpret_cast<uint4 *>(dst) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
  } else if constexpr (EPI == kEpiLogits) {
    for (int n = n0 + warp; n < n1; n += kThreads / 32) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int r = lane; r < kTileRows; r += 32) {
        const int row = row0 + r;
        if (row >= P.rows) break;
        const float v = stage[(n - n0) * kTileRows + r];
        if (P.y != nullptr) P.y[static_cast<size_t>(n) * P.rows + row] = v;
        if (argmax_better(v, row, bv, bi)) {
          bv = v;
          bi = row;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, ov, oi);
      }
      if (lane == 0) {
        P.part_val[static_cast<size_t>(tile) * P.pstride + n] = bv;
        P.part_idx[static_cast<size_t>(tile) * P.pstride + n] = bi;
      }
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ GemmParams P) {
  extern __shared__ __align__(1024) uint8_t smem[];
  // kEpiResid: the residual of the columns this CTA finishes, bulk-copied
  // while the MMAs run
  __shared__ __align__(128) __nv_bfloat16 s_res[EPI == kEpiResid ? kResPre * kTileRows : 8];
  __shared__ __align__(8) uint64_t s_resbar;
  // kEpiQkv: the columns' rows metadata and RoPE values, read before the
  // dependency wait (host-uploaded rows, constant tables)
  __shared__ int s_pos[EPI == kEpiQkv ? kMaxN : 1], s_slot[EPI == kEpiQkv ? kMaxN : 1];
  __shared__ float s_cs[EPI == kEpiQkv ? kResPre * 64 : 1];
  const int S = P.stages;
  uint8_t *sa = smem;                                                   // [S][16 KB]
  uint8_t *sb = smem + static_cast<size_t>(S) * kAStageBytes;           // [S][npad * 128]
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + gemm_data_bytes(S, P.npad, P.ksplit));
  uint64_t *empty = full + S;
  uint64_t *done = empty + S;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x / P.ksplit, split = blockIdx.x - tile * P.ksplit;
  const uint32_t ncols = tmem_cols(P.npad);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(done, 1);
    if (EPI == kEpiResid) mbar_init(&s_resbar, 1);
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
  grid_dep_launch();

  const int k0 = split * P.kst / P.ksplit;
  const int nk = (split + 1) * P.kst / P.ksplit - k0;  // K stages of this slice (>= 1)
  // the columns this CTA finishes: a share of them with K slices, else all
  const int n0 = P.ksplit > 1 ? split * P.N / P.ksplit : 0;
  const int n1 = P.ksplit > 1 ? (split + 1) * P.N / P.ksplit : P.N;
  const int res_cols = EPI == kEpiResid ? min(n1 - n0, kResPre) : 0;
  const int res_rows = min(kTileRows, P.rows - tile * kTileRows);

  if (warp == 0 && lane == 0) {
    // producer: a stage is one box of W's tile and one of the batch (full
    // boxes: row groups past either end arrive as zeros and still count).
    // The first stages' weights do not depend on earlier kernels: they are
    // requested before the wait for those kernels, the batch after it.
    const uint32_t bytes = kAStageBytes + static_cast<uint32_t>(P.npad) * 128;
    const int early = min(S, nk);
    for (int i = 0; i < early; ++i) {
      mbar_arrive_expect_tx(&full[i], bytes);
      tma_load_3d(sa + static_cast<size_t>(i) * kAStageBytes, &P.map_w, 0, k0 + i, tile * 16, &full[i]);
    }
    grid_dep_wait();
    for (int i = 0; i < early; ++i)
      tma_load_3d(sb + static_cast<size_t>(i) * P.npad * 128, &P.map_x, 0, k0 + i, 0, &full[i]);
    int issued = early;
    for (int i = early; i < nk; ++i) {
      const int s = i % S;
      const uint32_t ph = static_cast<uint32_t>(i / S) & 1u;
      if (!mbar_wait(&empty[s], ph ^ 1u, P.ctrl, P.limit_ns, kWhereEmpty)) break;
      mbar_arrive_expect_tx(&full[s], bytes);
      tma_load_3d(sa + static_cast<size_t>(s) * kAStageBytes, &P.map_w, 0, k0 + i, tile * 16, &full[s]);
      tma_load_3d(sb + static_cast<size_t>(s) * P.npad * 128, &P.map_x, 0, k0 + i, 0, &full[s]);
      ++issued;
    }
    // every load issued has landed before the CTA can exit
    for (int i = max(0, issued - S); i < issued; ++i)
      mbar_wait_quiet(&full[i % S], static_cast<uint32_t>(i / S) & 1u, P.limit_ns);
  } else {
    if constexpr (EPI == kEpiQkv) {
      // warps 2 and 3 of a tile with k / v rows: each column's position and
      // slot, then (lanes = dimensions) its RoPE cos / sin
      if (warp >= 2 && (tile + 1) * kTileRows > P.kv.QH * kHeadDimTc) {
        for (int c = threadIdx.x - 64; c < n1 - n0; c += 64) {
          s_pos[c] = P.R.pos[n0 + c];
          s_slot[c] = P.R.slot[n0 + c];
        }
        // warp 2 takes the even columns < kResPre, warp 3 the odd ones: lane k
        // fetches the position of the warp's column k, then every lane loads
        // its dimension of all the warp's columns, all loads in flight
        constexpr int kPer = kResPre / 2;
        const int cols = min(n1 - n0, kResPre);
        const int cl = warp - 2 + 2 * lane;
        const int pl = lane < kPer && cl < cols ? P.R.pos[n0 + cl] : 0;
        float cv[kPer], sv[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          const int p = __shfl_sync(0xffffffffu, pl, k);
          const bool in = warp - 2 + 2 * k < cols;
          cv[k] = in ? P.kv.cos[p * 32 + lane] : 0.f;
          sv[k] = in ? P.kv.sin[p * 32 + lane] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          const int c = warp - 2 + 2 * k;
          if (c < cols) {
            s_cs[c * 64 + lane] = cv[k];
            s_cs[c * 64 + 32 + lane] = sv[k];
          }
        }
      }
    }
    grid_dep_wait();  // the epilogue reads what earlier kernels wrote
    if (EPI == kEpiResid && warp == 2 && lane == 0 && res_cols > 0) {
      // the staged residual: one 16-byte-aligned run of the tile's rows per
      // column (rows a multiple of 8)
      const uint32_t bytes = static_cast<uint32_t>(res_rows) * 2;
      mbar_arrive_expect_tx(&s_resbar, bytes * static_cast<uint32_t>(res_cols));
      for (int c = 0; c < res_cols; ++c)
        bulk_g2s(s_res + c * kTileRows, P.resid + static_cast<size_t>(n0 + c) * P.rows + tile * kTileRows, bytes,
                 &s_resbar);
    }
    if (warp == 1 && lane == 0) {
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
          umma_bf16(tmem, smem_desc(a + kk * 256, 128, kGroupStageBytes),
                    smem_desc(b + kk * 256, 128, kGroupStageBytes), idesc, (i | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);  // the slot is free once these MMAs have read it
      }
      umma_commit(done);  // also on an early exit: nothing in flight when TMEM is freed
    }
  }
  __syncwarp();
  // epilogue: wait for the accumulator (or, after an abort, for the MMAs in
  // flight) and the staged residual
  const bool ok = __syncthreads_and(mbar_wait(done, 0, P.ctrl, P.limit_ns, kWhereFull) &&
                                    (res_cols == 0 || mbar_wait(&s_resbar, 0, P.ctrl, P.limit_ns, kWhereFull)) &&
                                    ld_volatile_int(&P.ctrl->abort) == 0) != 0;
  // no staged copy is in flight when the CTA exits (after an abort too)
  if (res_cols > 0 && warp == 2 && lane == 0) mbar_wait_quiet(&s_resbar, 0, P.limit_ns);
  tc_fence_after();
  const int r_t = warp * 32 + lane;  // this thread's row within the tile (its TMEM lane)
  const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  // the ring is idle now (every copy landed, every MMA done): its space
  // stages the tile's FP32 results (this slice's partial) [npad][128]
  float *stage = reinterpret_cast<float *>(smem);
  if (ok) {
    for (int c0 = 0; c0 < P.npad; c0 += 16) {
      uint32_t v[16];
      tmem_ld16(taddr + c0, v);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) stage[(c0 + j) * kTileRows + r_t] = __uint_as_float(v[j]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ncols);
  if (P.ksplit == 1) {
    if (ok) finish_tile<EPI>(P, stage, tile, 0, P.N, EpiSmem{s_res, s_pos, s_slot, s_cs});
    return;
  }
  // K slices: the tile's slices are one cluster (rank = slice).  Once every
  // partial is staged, slice s sums columns [s N / ksplit, (s + 1) N /
  // ksplit) -- a contiguous block of each slice's partial, read as 16-byte
  // vectors through distributed shared memory, every load in flight at once
  // -- in slice order (the result does not depend on which slice finishes
  // first) and finishes them.  Every CTA reaches both cluster barriers, on
  // an abort too, and none exits while a peer may still read its partial.
  cluster_arrive();
  cluster_wait();
  float *red = stage + static_cast<size_t>(P.npad) * kTileRows;
  if (ok) {
    const uint32_t base = smem_u32(stage) + static_cast<uint32_t>(n0 * kTileRows * 4);
    const int vecs = (n1 - n0) * (kTileRows / 4);  // float4s in the block
    constexpr int kPer = 4;                          // float4s per thread per pass
    for (int v0 = 0; v0 < vecs; v0 += kPer * kThreads) {
      float4 acc[kPer];
#pragma unroll
      for (int u = 0; u < kPer; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int sl = 0; sl < kMaxSlices; ++sl) {
        if (sl >= P.ksplit) break;
        const uint32_t peer = cluster_addr(base, static_cast<uint32_t>(sl));
        float4 v[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
          const int idx = v0 + u * kThreads + threadIdx.x;
          v[u] = idx < vecs ? ld_cluster_f32x4(peer + static_cast<uint32_t>(idx) * 16u) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
          acc[u].x += v[u].x;
          acc[u].y += v[u].y;
          acc[u].z += v[u].z;
          acc[u].w += v[u].w;
        }
      }
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int idx = v0 + u * kThreads + threadIdx.x;
        if (idx < vecs) reinterpret_cast<float4 *>(red)[idx] = acc[u];
      }
    }
  }
  cluster_arrive();
  __syncthreads();
  if (ok) finish_tile<EPI>(P, red, tile, n0, n1, EpiSmem{s_res, s_pos, s_slot, s_cs});
  cluster_wait();
}

// ---- persistent LM head -----------------------------------------------------------
// logits[n][r] = sum_k W[r][k] X[n][k] over the whole vocabulary with each
// tile's per-column maximum (np.argmax order) for argmax_reduce_kernel.
// One CTA per SM walks tiles blockIdx.x, blockIdx.x + gridDim.x, ...: warp 0
// lane 0 streams every (tile, K stage) of the CTA through one ring without
// a break between tiles, warp 1 lane 0 accumulates tile t into TMEM buffer
// t & 1, and warps 2..5 (TMEM lane quarters 2, 3, 0, 1) read a finished
// buffer -- the optional FP32 logits, then the tile transposed through
// shared memory and one thread per column scanning its 128 rows -- while
// the next tile's MMAs run.  (A shuffle reduction per column, unrolled over
// the columns, is tens of KB of code that misses the instruction cache on
// every pass; the scan loop is a few instructions.)
constexpr int kHeadThreads = 192;
constexpr int kHeadEpiWarps = 4;

__host__ __device__ inline size_t head_ring_bytes(int stages, int npad) {
  return static_cast<size_t>(stages) * (kAStageBytes + static_cast<size_t>(npad) * 128);
}
constexpr int kHeadStride = kTileRows + 1;  // transposed tile row pitch (floats): conflict-free
// ring | full[S] empty[S] acc_full[2] acc_empty[2] done | tmem slot | tile [npad][129] FP32
__host__ __device__ inline size_t head_smem_bytes(int stages, int npad) {
  return head_ring_bytes(stages, npad) + 8 * (2 * static_cast<size_t>(stages) + 5) + 16 +
         static_cast<size_t>(npad) * kHeadStride * 4;
}

// One row of a column scan whose rows arrive in index order: a larger value
// wins, a tie keeps the earlier row, a NaN beats every number and the first
// NaN stays (np.argmax order).
__device__ __forceinline__ void scan_take(float v, int i, float &bv, int &bi) {
  if (v > bv || (v != v && bv == bv)) {
    bv = v;
    bi = i;
  }
}

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// Named barrier over `threads` threads that also ANDs `pred` across them.
__device__ __forceinline__ bool named_and(int id, int threads, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, r;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred r, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, r;\n\t}"
      : "=r"(out)
      : "r"(pred ? 1u : 0u), "r"(id), "r"(threads)
      : "memory");
  return out != 0;
}

__global__ void __launch_bounds__(kHeadThreads, 1) lm_head_kernel(const __grid_constant__ GemmParams P) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int S = P.stages;
  uint8_t *sa = smem;
  uint8_t *sb = smem + static_cast<size_t>(S) * kAStageBytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + head_ring_bytes(S, P.npad));
  uint64_t *empty = full + S;
  uint64_t *acc_full = empty + S;    // [2] an accumulator buffer holds a finished tile
  uint64_t *acc_empty = acc_full + 2;  // [2] the epilogue has read it
  uint64_t *done = acc_empty + 2;      // every MMA of this CTA has completed
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  float *tpose = reinterpret_cast<float *>(tmem_slot + 4);  // [npad][kHeadStride]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ncols = tmem_cols(2 * P.npad);
  const int mine = (P.tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                   static_cast<int>(gridDim.x);  // tiles of this CTA
  const int total = mine * P.kst;                // (tile, K stage) steps

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kHeadEpiWarps);
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
  grid_dep_launch();

  if (warp == 0) {
    if (lane == 0) {
      // producer; the first stages' weights are requested before the wait
      // for the previous kernel, the batch rows after it
      const uint32_t bytes = kAStageBytes + static_cast<uint32_t>(P.npad) * 128;
      const int early = min(S, total);
      for (int it = 0; it < early; ++it) {
        const int tile = static_cast<int>(blockIdx.x) + (it / P.kst) * static_cast<int>(gridDim.x);
        mbar_arrive_expect_tx(&full[it], bytes);
        tma_load_3d(sa + static_cast<size_t>(it) * kAStageBytes, &P.map_w, 0, it % P.kst, tile * 16, &full[it]);
      }
      grid_dep_wait();
      for (int it = 0; it < early; ++it)
        tma_load_3d(sb + static_cast<size_t>(it) * P.npad * 128, &P.map_x, 0, it % P.kst, 0, &full[it]);
      int issued = early;
      for (int it = early; it < total; ++it) {
        const int s = it % S;
        const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, P.ctrl, P.limit_ns, kWhereEmpty)) break;
        const int tile = static_cast<int>(blockIdx.x) + (it / P.kst) * static_cast<int>(gridDim.x);
        mbar_arrive_expect_tx(&full[s], bytes);
        tma_load_3d(sa + static_cast<size_t>(s) * kAStageBytes, &P.map_w, 0, it % P.kst, tile * 16, &full[s]);
        tma_load_3d(sb + static_cast<size_t>(s) * P.npad * 128, &P.map_x, 0, it % P.kst, 0, &full[s]);
        ++issued;
      }
      for (int it = max(0, issued - S); it < issued; ++it)
        mbar_wait_quiet(&full[it % S], static_cast<uint32_t>(it / S) & 1u, P.limit_ns);
    }
  } else if (warp == 1) {
    grid_dep_wait();
    if (lane == 0) {
      // MMA issuer: tile t into TMEM columns [(t & 1) npad, + npad)
      const uint32_t idesc = idesc_bf16(P.npad);
      bool go = true;
      for (int t = 0; t < mine && go; ++t) {
        const int buf = t & 1;
        if (t >= 2 && !mbar_wait(&acc_empty[buf], static_cast<uint32_t>((t >> 1) - 1) & 1u, P.ctrl, P.limit_ns,
                                 kWhereEmpty))
          break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * P.npad);
        for (int k = 0; k < P.kst; ++k) {
          const int it = t * P.kst + k;
          const int s = it % S;
          if (!mbar_wait(&full[s], static_cast<uint32_t>(it / S) & 1u, P.ctrl, P.limit_ns, kWhereFull)) {
            go = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(sa + static_cast<size_t>(s) * kAStageBytes);
          const uint32_t b = smem_u32(sb + static_cast<size_t>(s) * P.npad * 128);
#pragma unroll
          for (int kk = 0; kk < kStageK / 16; ++kk)
            umma_bf16(d, smem_desc(a + kk * 256, 128, kGroupStageBytes), smem_desc(b + kk * 256, 128, kGroupStageBytes),
                      idesc, (k | kk) != 0 ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (go) umma_commit(&acc_full[buf]);
      }
      umma_commit(done);  // also on an early exit: nothing in flight when TMEM is freed
    }
  } else {

    // epilogue warps 2..5: warp w reads TMEM lanes 32 (w % 4) .. + 31
    grid_dep_wait();
    const int q = warp & 3;
    int parts = 32;  // threads per column in the scan: 128 / (N rounded up to a power of two), at most 32
    while (parts > 1 && (128 / parts) < P.N) parts >>= 1;
    for (int t = 0; t < mine; ++t) {
      const int buf = t & 1;
      // the four warps agree before any of them waits at a named barrier
      if (!named_and(1, kHeadEpiWarps * 32,
                     mbar_wait(&acc_full[buf], static_cast<uint32_t>(t >> 1) & 1u, P.ctrl, P.limit_ns, kWhereFull)))
        break;
      tc_fence_after();
      const int tile = static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x);
      const int row = tile * kTileRows + q * 32 + lane;
      const bool valid = row < P.rows;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * P.npad);
      for (int c0 = 0; c0 < P.N; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(taddr + c0, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float val = __uint_as_float(v[j]);
          if (valid && c0 + j < P.N && P.y != nullptr) P.y[static_cast<size_t>(c0 + j) * P.rows + row] = val;
          tpose[(c0 + j) * kHeadStride + q * 32 + lane] = val;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_count(&acc_empty[buf], 1);  // the buffer may take the next tile
      named_sync(1, kHeadEpiWarps * 32);
      // the column maxima: a column's 128 rows split over `parts` threads
      // of one warp, each walking rows part, part + parts, ... in four
      // interleaved chains, then a butterfly over the column's threads
      const int live = min(kTileRows, P.rows - tile * kTileRows);  // rows of this tile inside W
      const int et = (warp - 2) * 32 + lane;  // epilogue thread
      const int n = et / parts, part = et - n * parts;
      const int row0 = tile * kTileRows;
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      if (n < P.N) {
        const float *col = tpose + n * kHeadStride;
        float cv[4];
        int ci[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // each chain starts at its first row: a tie keeps the earlier row
          const int r = part + c * parts;
          cv[c] = r < live ? col[r] : -INFINITY;
          ci[c] = r < live ? row0 + r : 0x7fffffff;
        }
        for (int r = part + 4 * parts; r < live; r += 4 * parts) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int rr = r + c * parts;
            if (rr < live) scan_take(col[rr], row0 + rr, cv[c], ci[c]);
          }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) argmax_merge(bv, bi, cv[c], ci[c]);
      }
      for (int o = parts / 2; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, ov, oi);
      }
      if (n < P.N && part == 0) {
        P.part_val[static_cast<size_t>(tile) * P.pstride + n] = bv;
        P.part_idx[static_cast<size_t>(tile) * P.pstride + n] = bi;
      }
      named_sync(1, kHeadEpiWarps * 32);  // the transposed tile may be overwritten
    }
  }
  __syncthreads();
  if (warp == 0) {
    mbar_wait_quiet(done, 0, P.limit_ns);
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
}

// ---- per-row kernels of the batched step ---------------------------------------
// Row n of out (packed row-group layout) = bf16((x * inv_rms) * gamma) of
// row rows[n] of x, or of row n when rows is NULL, for the n < count rows;
// a warp per row, 4 rows per CTA.
__global__ void __launch_bounds__(kThreads) norm_pack_kernel(const __nv_bfloat16 *x, const int *rows, int count,
                                                             const float *gamma, float eps, int H, uint8_t *out) {
  grid_dep_launch();
  grid_dep_wait();
  const int n = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  if (n >= count) return;
  norm_pack_row(x + static_cast<size_t>(rows ? rows[n] : n) * H, gamma, eps, H, out, n);
}

// For the n < count rows: h[n][:] = the embedding row of token tok[n]
// (generate.py:758-768) and row n of out = its RMS norm with the first
// layer's gamma; a warp per row, 4 rows per CTA.
__global__ void __launch_bounds__(kThreads) embed_norm_kernel(const __nv_bfloat16 *embed, const int *tok, int count,
                                                              const float *gamma, float eps, int H,
                                                              __nv_bfloat16 *h, uint8_t *out) {
  grid_dep_launch();
  grid_dep_wait();
  const int n = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (n >= count) return;
  const __nv_bfloat16 *src = embed + static_cast<size_t>(tok[n]) * H;
  uint4 *dst = reinterpret_cast<uint4 *>(h + static_cast<size_t>(n) * H);
  for (int i = lane; i < H / 8; i += 32) dst[i] = __ldg(reinterpret_cast<const uint4 *>(src) + i);
  norm_pack_row(src, gamma, eps, H, out, n);
}

// Attention of every (row, q head): a CTA per (row, kv head) copies that kv
// head's K / V rows 0..pos into shared memory; warp w attends q head
// j * group + w with attend_warp() and writes its 64 outputs into the
// o-projection's packed input.
__global__ void attention_kernel(const __grid_constant__ KvArgs A, Rows R, uint8_t *att) {
  extern __shared__ __align__(128) uint8_t sm[];
  grid_dep_launch();
  const int n = blockIdx.x, j = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the rows' metadata (uploaded before the step's first kernel) and the
  // RoPE tables do not depend on the kernels before this one: read before
  // the wait
  const int p = R.pos[n], slot = R.slot[n];
  const float rc = A.cos[p * 32 + lane], rs = A.sin[p * 32 + lane];
  // K / V rows of the slot's positions before its first row in this step
  // were written by earlier steps: they are fetched before the wait, the
  // rest (this step's qkv kernel writes them) after it
  __shared__ int s_first;
  if (threadIdx.x == 0) s_first = p;
  __syncthreads();
  for (int i = threadIdx.x; i < static_cast<int>(gridDim.x); i += blockDim.x)
    if (R.slot[i] == slot) atomicMin(&s_first, R.pos[i]);
  __syncthreads();
  uint8_t *kb = sm, *vb = sm + static_cast<size_t>(A.ctx) * 128;
  float *qf = reinterpret_cast<float *>(sm + static_cast<size_t>(2) * A.ctx * 128) + warp * 128;
  const int pieces = (p + 1) * 8;  // 16-byte pieces of positions 0..p
  const int early = s_first * 8;   // pieces of positions < s_first (<= p)
  const uint8_t *ks = kv_rows(A, slot, j, 0), *vs = kv_rows(A, slot, j, 1);
  for (int i = threadIdx.x; i < 2 * early; i += blockDim.x) {
    const int kind = i >= early ? 1 : 0, off = (i - kind * early) * 16;
    cp_async16((kind ? vb : kb) + off, (kind ? vs : ks) + off);
  }
  grid_dep_wait();
  const int late = pieces - early;
  for (int i = threadIdx.x; i < 2 * late; i += blockDim.x) {
    const int kind = i >= late ? 1 : 0, off = (early + i - kind * late) * 16;
    cp_async16((kind ? vb : kb) + off, (kind ? vs : ks) + off);
  }
  cp_async_commit();
  const int h = j * A.group + warp;
  const uint32_t *row = reinterpret_cast<const uint32_t *>(A.qkv + static_cast<size_t>(n) * A.QKV);
  __nv_bfloat16 lo, hi;
  rope_pair_cs(row + h * 32, lane, rc, rs, lo, hi);
  qf[lane] = bf2f(lo);
  qf[lane + 32] = bf2f(hi);
  cp_async_wait_all();
  __syncthreads();
  const uint32_t o = attend_warp(qf, qf + 64, kb, vb, p);
  const int c = h * 64 + 2 * lane;  // output column of this lane's pair
  *reinterpret_cast<uint32_t *>(att + (static_cast<size_t>(n >> 3) * (A.H / 8) + (c >> 3)) * 128 + (n & 7) * 16 +
                                (c & 7) * 2) = o;
}

// out[n] = argmax over the LM head's tiles of row n (np.argmax order).
__global__ void argmax_reduce_kernel(const float *pv, const int *pi, int tiles, int pstride, int *out) {
  __shared__ float sv[8];
  __shared__ int si[8];
  grid_dep_launch();
  grid_dep_wait();
  const int n = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int t = threadIdx.x; t < tiles; t += blockDim.x)
    argmax_merge(bv, bi, pv[static_cast<size_t>(t) * pstride + n], pi[static_cast<size_t>(t) * pstride + n]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_merge(bv, bi, ov, oi);
  }
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x / 32); ++w) argmax_merge(bv, bi, sv[w], si[w]);
    out[n] = bi;
  }
}

}  // namespace tc
}  // namespace hb
