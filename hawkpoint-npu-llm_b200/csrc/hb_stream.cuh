// hb_stream.cuh -- the weight stream shared by the decoder and GEMV kernels.
//
// Each CTA owns a contiguous run of row groups of every projection it works
// on.  One producer thread copies that run, chunk by chunk, into a ring of
// shared-memory slots with cp.async.bulk (completion on a per-slot "full"
// mbarrier); the consumer warps compute on a slot and release it on its
// "empty" mbarrier.  The producer never waits on activations, so it keeps
// streaming weights for the next phases while the consumers wait at a grid
// barrier: the barrier latency hides under the HBM stream.
//
// Packed projection layout (runtime/layout.py): row group g (8 rows) at
// g * kc * 128 bytes, then chunk column j (16 bytes of each of the 8 rows) at
// j * 128 + r * 16.  A chunk is either several whole row groups or, when one
// row group is larger than a slot, a K-slice of kPartCols chunk columns.
#pragma once

#include "hb_device.cuh"

namespace hb {

constexpr int kWarps = 8;                  // consumer warps
constexpr int kConsumerThreads = kWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;  // + producer warp
constexpr uint32_t kSlotBytes = 16384;
constexpr int kPartCols = 128;             // chunk columns per K-slice (kSlotBytes / 128)
constexpr int kColGroups = kWarps * 4;     // split-K column groups per CTA

struct MatRange {
  const uint8_t *base;  // row group 0 of the matrix
  int g0, g1;           // row-group range owned by this CTA
  int kc;               // 16-byte chunk columns per row
};

__device__ __forceinline__ int rg_per_chunk(int kc) {
  const int rgb = kc * 128;
  return rgb <= static_cast<int>(kSlotBytes) ? static_cast<int>(kSlotBytes) / rgb : 0;
}

__device__ __forceinline__ int parts_per_rg(int kc) { return (kc + kPartCols - 1) / kPartCols; }

__device__ __forceinline__ int num_chunks(const MatRange &r) {
  const int n = r.g1 - r.g0;
  if (n <= 0 || r.base == nullptr) return 0;
  const int rpc = rg_per_chunk(r.kc);
  if (rpc > 0) return (n + rpc - 1) / rpc;
  return n * parts_per_rg(r.kc);
}

struct ChunkInfo {
  const uint8_t *src;
  uint32_t bytes;
  int rg;         // first row group
  int nrg;        // row groups in the chunk
  int col0;       // first chunk column
  int ncols;      // chunk columns per row group in the chunk
  bool last_part; // the chunk ends its row group(s)
};

__device__ __forceinline__ ChunkInfo chunk_info(const MatRange &r, int t) {
  ChunkInfo c;
  const int rpc = rg_per_chunk(r.kc);
  const size_t rgb = static_cast<size_t>(r.kc) * 128;
  if (rpc > 0) {
    c.rg = r.g0 + t * rpc;
    c.nrg = min(rpc, r.g1 - c.rg);
    c.col0 = 0;
    c.ncols = r.kc;
    c.last_part = true;
    c.src = r.base + static_cast<size_t>(c.rg) * rgb;
    c.bytes = static_cast<uint32_t>(c.nrg * rgb);
  } else {
    const int ppr = parts_per_rg(r.kc);
    const int q = t / ppr, p = t - q * ppr;
    c.rg = r.g0 + q;
    c.nrg = 1;
    c.col0 = p * kPartCols;
    c.ncols = min(kPartCols, r.kc - c.col0);
    c.last_part = (p == ppr - 1);
    c.src = r.base + static_cast<size_t>(c.rg) * rgb + static_cast<size_t>(c.col0) * 128;
    c.bytes = static_cast<uint32_t>(c.ncols * 128);
  }
  return c;
}

// Balanced contiguous split of n units over parts.
__device__ __forceinline__ int split_lo(int n, int parts, int idx) {
  return static_cast<int>((static_cast<long long>(n) * idx) / parts);
}

// Shared-memory ring state of one CTA.
struct Ring {
  uint8_t *slots;
  uint64_t *full;
  uint64_t *empty;
  int nslots;
  uint32_t counter;  // chunks consumed so far in this launch (per thread copy)
};

// Producer: issue every chunk of `r` in order.  Returns false on abort.
__device__ __forceinline__ bool produce_range(Ring &ring, const MatRange &r, uint32_t &issued,
                                              Ctrl *ctrl, uint64_t limit_ns, uint64_t policy) {
  const int n = num_chunks(r);
  for (int t = 0; t < n; ++t) {
    const int slot = static_cast<int>(issued % ring.nslots);
    const uint32_t use = issued / ring.nslots;
    if (use > 0 && !mbar_wait(&ring.empty[slot], (use - 1) & 1u, ctrl, limit_ns, kWhereEmpty))
      return false;
    const ChunkInfo c = chunk_info(r, t);
    mbar_arrive_expect_tx(&ring.full[slot], c.bytes);
    bulk_g2s_evict_first(ring.slots + static_cast<size_t>(slot) * kSlotBytes, c.src, c.bytes,
                         &ring.full[slot], policy);
    ++issued;
  }
  return true;
}

// Producer exit: wait until every issued copy has landed, so no bulk copy
// still targets this CTA's shared memory when it exits.
__device__ __forceinline__ void drain_ring(Ring &ring, uint32_t issued, Ctrl *ctrl) {
  const uint32_t first = issued > static_cast<uint32_t>(ring.nslots) ? issued - ring.nslots : 0;
  for (uint32_t i = first; i < issued; ++i) {
    const int slot = static_cast<int>(i % ring.nslots);
    const uint32_t parity = (i / ring.nslots) & 1u;
    const uint64_t start = globaltimer_ns();
    while (!mbar_try_wait(&ring.full[slot], parity)) {
      if (globaltimer_ns() - start > 2000000000ull) {
        raise_error(ctrl, kErrTimeout, kWhereDrain);
        break;
      }
    }
  }
}

// Consumer: wait for the next chunk.
__device__ __forceinline__ bool ring_acquire(Ring &ring, uint32_t g, Ctrl *ctrl, uint64_t limit_ns,
                                             const uint8_t *&slot_ptr, int &slot) {
  slot = static_cast<int>(g % ring.nslots);
  slot_ptr = ring.slots + static_cast<size_t>(slot) * kSlotBytes;
  return mbar_wait(&ring.full[slot], (g / ring.nslots) & 1u, ctrl, limit_ns, kWhereFull);
}

// Activation vector element loads from shared memory (BF16 [K] per batch row).
template <bool W8>
struct XLoad;

template <>
struct XLoad<false> {
  // chunk column = 8 BF16 activations
  __device__ __forceinline__ static float dot(const uint4 w, const __nv_bfloat16 *x, int col,
                                              float acc) {
    const uint4 xv = *reinterpret_cast<const uint4 *>(x + col * 8);
    return dot8_bf16(w, xv, acc);
  }
};

template <>
struct XLoad<true> {
  // chunk column = 16 int8 weights = 16 activations
  __device__ __forceinline__ static float dot(const uint4 w, const __nv_bfloat16 *x, int col,
                                              float acc) {
    const uint4 x0 = *reinterpret_cast<const uint4 *>(x + col * 16);
    const uint4 x1 = *reinterpret_cast<const uint4 *>(x + col * 16 + 8);
    return dot16_i8(w, x0, x1, acc);
  }
};

// Split-K consumption of a row-group range by all consumer warps.  Every
// warp sees every chunk; column group cg = warp*4 + lane/8 takes chunk columns
// cg, cg+32, ... (chunk-column offsets of K-slices are multiples of 32, so a
// lane keeps the same columns across the slices of one row group).  The
// per-warp partial of (batch row m, local row) goes to
// red[(warp * MB + m) * red_rows + local_row]; the caller sums the warps
// after a consumer_sync.  xs: BF16 activations [MB][K] in shared memory.
template <int MB, bool W8>
__device__ __forceinline__ bool consume_splitk(Ring &ring, const MatRange &r,
                                               const __nv_bfloat16 *xs, int K, int mrows,
                                               float *red, int red_rows, Ctrl *ctrl,
                                               uint64_t limit_ns) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rr = lane & 7;
  const int cg = warp * 4 + (lane >> 3);
  const int n = num_chunks(r);
  float acc[MB];
#pragma unroll
  for (int m = 0; m < MB; ++m) acc[m] = 0.f;
  for (int t = 0; t < n; ++t) {
    const uint8_t *s;
    int slot;
    if (!ring_acquire(ring, ring.counter++, ctrl, limit_ns, s, slot)) return false;
    const ChunkInfo c = chunk_info(r, t);
    for (int q = 0; q < c.nrg; ++q) {
      const uint8_t *sg = s + static_cast<size_t>(q) * c.ncols * 128 + rr * 16;
      for (int j = cg; j < c.ncols; j += kColGroups) {
        const uint4 w = *reinterpret_cast<const uint4 *>(sg + j * 128);
        const int col = c.col0 + j;
#pragma unroll
        for (int m = 0; m < MB; ++m)
          if (m < mrows) acc[m] = XLoad<W8>::dot(w, xs + static_cast<size_t>(m) * K, col, acc[m]);
      }
      if (c.last_part) {
        const int local = (c.rg + q - r.g0) * 8 + rr;
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          float v = acc[m];
          v += __shfl_xor_sync(0xffffffffu, v, 8);
          v += __shfl_xor_sync(0xffffffffu, v, 16);
          if (lane < 8 && m < mrows) red[(warp * MB + m) * red_rows + local] = v;
          acc[m] = 0.f;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive_count(&ring.empty[slot], 1);
  }
  return true;
}

// Row-group-per-warp consumption (small K): every warp waits for every chunk,
// warp w takes row groups w, w+8, ... of it; lane/8 strides the columns.
// on_row(m, row, value) runs on lanes 0..7 with the full dot product.
template <int MB, bool W8, class F>
__device__ __forceinline__ bool consume_rg_per_warp(Ring &ring, const MatRange &r,
                                                    const __nv_bfloat16 *xs, int K, int mrows,
                                                    Ctrl *ctrl, uint64_t limit_ns, F &&on_row) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rr = lane & 7, cq = lane >> 3;
  const int n = num_chunks(r);
  for (int t = 0; t < n; ++t) {
    const uint8_t *s;
    int slot;
    if (!ring_acquire(ring, ring.counter++, ctrl, limit_ns, s, slot)) return false;
    const ChunkInfo c = chunk_info(r, t);
    for (int q = warp; q < c.nrg; q += kWarps) {
      const uint8_t *sg = s + static_cast<size_t>(q) * c.ncols * 128 + rr * 16;
      float acc[MB];
#pragma unroll
      for (int m = 0; m < MB; ++m) acc[m] = 0.f;
      for (int j = cq; j < c.ncols; j += 4) {
        const uint4 w = *reinterpret_cast<const uint4 *>(sg + j * 128);
#pragma unroll
        for (int m = 0; m < MB; ++m)
          if (m < mrows) acc[m] = XLoad<W8>::dot(w, xs + static_cast<size_t>(m) * K, c.col0 + j, acc[m]);
      }
      const int row = (c.rg + q) * 8 + rr;
#pragma unroll
      for (int m = 0; m < MB; ++m) {
        float v = acc[m];
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        if (lane < 8 && m < mrows) on_row(m, row, v);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive_count(&ring.empty[slot], 1);
  }
  return true;
}

// Chunk-per-warp consumption (throughput mode, whole row groups per chunk):
// chunk t goes to warp t % 8, which releases it alone (arrival count 8).
template <int MB, bool W8, class F>
__device__ __forceinline__ bool consume_chunk_per_warp(Ring &ring, const MatRange &r,
                                                       const __nv_bfloat16 *xs, int K, int mrows,
                                                       Ctrl *ctrl, uint64_t limit_ns, F &&on_row) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rr = lane & 7, cq = lane >> 3;
  const int n = num_chunks(r);
  const uint32_t base = ring.counter;
  ring.counter += n;
  for (int t = warp; t < n; t += kWarps) {
    const uint8_t *s;
    int slot;
    if (!ring_acquire(ring, base + t, ctrl, limit_ns, s, slot)) return false;
    const ChunkInfo c = chunk_info(r, t);
    for (int q = 0; q < c.nrg; ++q) {
      const uint8_t *sg = s + static_cast<size_t>(q) * c.ncols * 128 + rr * 16;
      float acc[MB];
#pragma unroll
      for (int m = 0; m < MB; ++m) acc[m] = 0.f;
#pragma unroll 4
      for (int j = cq; j < c.ncols; j += 4) {
        const uint4 w = *reinterpret_cast<const uint4 *>(sg + j * 128);
#pragma unroll
        for (int m = 0; m < MB; ++m)
          if (m < mrows) acc[m] = XLoad<W8>::dot(w, xs + static_cast<size_t>(m) * K, c.col0 + j, acc[m]);
      }
      const int row = (c.rg + q) * 8 + rr;
#pragma unroll
      for (int m = 0; m < MB; ++m) {
        float v = acc[m];
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        if (lane < 8 && m < mrows) on_row(m, row, v);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive_count(&ring.empty[slot], kWarps);
  }
  return true;
}

}  // namespace hb
