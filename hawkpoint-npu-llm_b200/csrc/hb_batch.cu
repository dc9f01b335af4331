// hb_batch.cu -- the batched tensor-core path of libhawkb200.so.
//
// The persistent decoder kernel (hb_decoder.cuh) streams every weight once
// per launch for at most 8 rows on mma.sync.  Prefill (many positions of one
// sequence) and multi-stream decode (one position of many sequences) are
// dense contractions over many rows, so they run here instead as a short
// sequence of kernels per layer around tcgen05 GEMMs (hb_tc.cuh): the
// weights stream once per step for up to 128 rows, accumulate in TMEM, and
// the epilogues apply the reference's BF16 rounding points.
#include "hb_engine_impl.h"
#include "hb_tc.cuh"

using namespace hbi;

namespace {

// K slices per tile so that tiles x slices roughly fills the GPU, each slice
// at least two K stages when the matrix has them.
int choose_ksplit(int tiles, int kst, int sms) {
  int ks = (sms + tiles - 1) / tiles;
  ks = std::min(ks, kst >= 2 ? kst / 2 : 1);
  return std::max(ks, 1);
}

int choose_stages(int npad) {
  const size_t per = hb::tc::kAStageBytes + static_cast<size_t>(npad) * 128;
  const int s = static_cast<int>((200u * 1024u - 64u) / (per + 16));
  return std::max(2, std::min(6, s));
}

struct GemmShape {
  int tiles, ksplit, kst, npad, stages;
  size_t ws_floats;
};

GemmShape gemm_shape(int rows, int k, int n, int sms) {
  GemmShape g{};
  g.tiles = (rows + hb::tc::kTileRows - 1) / hb::tc::kTileRows;
  g.kst = k / hb::tc::kStageK;
  g.ksplit = choose_ksplit(g.tiles, g.kst, sms);
  g.npad = hb::tc::pad_n(n);
  g.stages = choose_stages(g.npad);
  g.ws_floats = g.ksplit > 1 ? static_cast<size_t>(g.tiles) * g.ksplit * g.npad * hb::tc::kTileRows : 0;
  return g;
}

constexpr size_t kCtrlBytes = 256;

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace

namespace hbi {
void batch_release(hb_engine *) {}
}  // namespace hbi

extern "C" {

size_t hb_tc_gemm_scratch_bytes(int rows, int k, int n) {
  if (rows <= 0 || k <= 0 || n <= 0) return 0;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaGetLastError();
  const GemmShape g = gemm_shape(rows, k, n, sms);
  return kCtrlBytes + align256(sizeof(unsigned int) * g.tiles) + g.ws_floats * sizeof(float);
}

int hb_tc_gemm(const void *w_dev, int rows, int k, const void *x_dev, int n, float *y_dev, void *scratch_dev,
               size_t scratch_bytes, void *stream) {
  if (!w_dev || !x_dev || !y_dev || !scratch_dev)
    return fail(nullptr, HB_ERR_INVALID_ARG, "hb_tc_gemm: null pointer");
  if (rows <= 0 || rows % 8 || k <= 0 || k % hb::tc::kStageK || n < 1 || n > hb::tc::kMaxN)
    return fail(nullptr, HB_ERR_INVALID_ARG,
                "hb_tc_gemm: rows must be a positive multiple of 8, k of 64, and 1 <= n <= 256");
  if ((reinterpret_cast<uintptr_t>(w_dev) | reinterpret_cast<uintptr_t>(x_dev) |
       reinterpret_cast<uintptr_t>(scratch_dev)) & 15)
    return fail(nullptr, HB_ERR_INVALID_ARG, "hb_tc_gemm: operands must be 16-byte aligned");
  int dev = 0, sms = 0, major = 0;
  HB_CUDA(nullptr, cudaGetDevice(&dev));
  HB_CUDA(nullptr, cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  HB_CUDA(nullptr, cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  if (major != 10) return fail(nullptr, HB_ERR_UNSUPPORTED, "hb_tc_gemm: needs an sm_100 GPU");
  const GemmShape g = gemm_shape(rows, k, n, sms);
  const size_t need = kCtrlBytes + align256(sizeof(unsigned int) * g.tiles) + g.ws_floats * sizeof(float);
  if (scratch_bytes < need)
    return fail(nullptr, HB_ERR_INVALID_ARG, "hb_tc_gemm: scratch needs %zu bytes", need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *scr = static_cast<uint8_t *>(scratch_dev);
  // control block and slice counters start at zero on every call
  HB_CUDA(nullptr, cudaMemsetAsync(scr, 0, kCtrlBytes + align256(sizeof(unsigned int) * g.tiles), st));
  hb::tc::GemmParams P{};
  P.w = static_cast<const uint8_t *>(w_dev);
  P.x = static_cast<const uint8_t *>(x_dev);
  P.rows = rows;
  P.K = k;
  P.N = n;
  P.npad = g.npad;
  P.tiles = g.tiles;
  P.ksplit = g.ksplit;
  P.kst = g.kst;
  P.stages = g.stages;
  P.y = y_dev;
  P.ctrl = reinterpret_cast<hb::Ctrl *>(scr);
  P.cnt = reinterpret_cast<unsigned int *>(scr + kCtrlBytes);
  P.ws = g.ws_floats ? reinterpret_cast<float *>(scr + kCtrlBytes + align256(sizeof(unsigned int) * g.tiles))
                     : nullptr;
  P.limit_ns = kDefaultLimitNs;
  const size_t smem = hb::tc::gemm_smem_bytes(g.stages, g.npad);
  HB_CUDA(nullptr, cudaFuncSetAttribute(hb::tc::gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)));
  hb::tc::gemm_kernel<<<g.tiles * g.ksplit, hb::tc::kThreads, smem, st>>>(P);
  HB_CUDA(nullptr, cudaGetLastError());
  return HB_OK;
}

int hb_tc_gemm_status(const void *scratch_dev, void *stream) {
  if (!scratch_dev) return fail(nullptr, HB_ERR_INVALID_ARG, "hb_tc_gemm_status: null scratch");
  hb::Ctrl c{};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  HB_CUDA(nullptr, cudaMemcpyAsync(&c, scratch_dev, sizeof(c), cudaMemcpyDeviceToHost, st));
  HB_CUDA(nullptr, cudaStreamSynchronize(st));
  if (c.err == hb::kErrTimeout)
    return fail(nullptr, HB_ERR_DEVICE_TIMEOUT, "hb_tc_gemm: a device wait gave up (where %d)", c.err_where);
  return c.err ? fail(nullptr, HB_ERR_STATE, "hb_tc_gemm: device error %d", c.err) : HB_OK;
}

}  // extern "C"
