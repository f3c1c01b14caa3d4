// tc_conv_w8a8_noalloc: the W8A8 convolution without any device allocation.
//
// The regular conv path (a conv descriptor through tc_run_queue) gathers the input windows into a
// scratch buffer that the library grows with cudaMalloc as needed. Some callers cannot let a
// library allocate device memory at call time: a serving process that has reserved all of HBM
// for its own allocator up front, an embedder that must keep a fixed, load-time-known device
// footprint, or a latency-critical loop that cannot afford the device-wide synchronisation that
// cudaMalloc / cudaFree may cause. This entry point serves them: the gather buffer is a fixed
// array in device global memory, so a call allocates nothing.
//
// Limits and sharing rules:
//   * the gathered matrix (OH*OW rows of KH*KW*Cin bytes) must fit kNoAllocScratch bytes;
//     larger requests return TC_ERR_TOO_LARGE before anything runs;
//   * every GPU that loads the library holds the array (kNoAllocScratch bytes) until exit;
//   * all calls on a device share the one array, and it keeps what the last call left in it.
//     Each call writes every byte it later reads (zero padding included), so nothing needs
//     clearing between calls, but two calls whose work overlaps on the GPU (different streams,
//     or different host threads without ordering) race on the array: order them on one stream.
//   * the first call on each device looks up the array's device address (cudaGetSymbolAddress)
//     with that device current; later calls reuse it. Under CUDA's lazy module loading (the
//     default) that first call is also what loads the array's module onto the device, so the
//     16 MiB are taken at the first call on a device, not when the library is loaded. Make that
//     first call before capturing a stream into a CUDA graph.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/tarscuda.h"
#include "ops.h"

namespace {

constexpr uint64_t kNoAllocScratch = 16ull << 20;   // 16 MiB per device
static __device__ __align__(256) uint8_t g_conv_scratch[kNoAllocScratch];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// The host-side name g_conv_scratch is only a stand-in for the device array; a kernel needs the
// address the runtime reports for the current device.
cudaError_t scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_conv_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" int tc_conv_w8a8_noalloc(const uint8_t* img, uint64_t ld, int32_t H, int32_t W, int32_t Cin, int32_t KH,
                                    int32_t KW, int32_t stride, int32_t pad, const uint8_t* weights,
                                    const float* scale, int32_t per_channel, const float* bias, uint8_t* y,
                                    uint64_t ldy, int32_t N, int32_t act, int32_t out, float out_scale,
                                    void* stream) {
  if (!img || !weights || !scale || !y || H <= 0 || W <= 0 || Cin <= 0 || KH <= 0 || KW <= 0 || stride <= 0 ||
      pad < 0 || pad >= KH || pad >= KW || N <= 0 || act < 0 || act > 7 || out < 0 || out > 2 || ld < (uint64_t)Cin)
    return TC_ERR_ARG;
  // every index the gather computes stays far inside 64 bits: at most 2^31 pixels
  if ((uint64_t)H * (uint64_t)W > (1ull << 31)) return TC_ERR_ARG;
  const int64_t HP = (int64_t)H + 2 * (int64_t)pad, WP = (int64_t)W + 2 * (int64_t)pad;
  if (HP < KH || WP < KW) return TC_ERR_ARG;
  const int64_t OH = (HP - KH) / stride + 1, OW = (WP - KW) / stride + 1;
  const uint64_t K = (uint64_t)KH * KW * Cin, M = (uint64_t)OH * (uint64_t)OW;
  if (K % 16 || M > 65535 || K > 65535 || ldy < (uint64_t)N * (out == 0 ? 4 : out == 1 ? 2 : 1)) return TC_ERR_ARG;
  if (M * K > kNoAllocScratch) return TC_ERR_TOO_LARGE;
  void* scratch = nullptr;
  if (scratch_for_current_device(&scratch) != cudaSuccess) return TC_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;

  tc::Im2colArgs ia{};
  ia.img = img; ia.ld = ld; ia.out = (uint8_t*)scratch;
  ia.H = H; ia.W = W; ia.KH = KH; ia.KW = KW; ia.S = stride; ia.P = pad; ia.Cin = Cin; ia.OH = (int)OH; ia.OW = (int)OW;
  if (tc::launch_im2col(ia, st) != cudaSuccess) return TC_ERR_CUDA;

  tc::GemmArgs g{};
  g.A = (const uint8_t*)scratch; g.lda = K;
  g.W = weights; g.scale = (const uint8_t*)scale; g.per_channel = per_channel != 0;
  g.srow = nullptr; g.bias = (const uint8_t*)bias;
  g.Y = y; g.ldy = ldy;
  g.M = (int)M; g.N = N; g.K = (int)K; g.act = act; g.out = out; g.out_scale = out_scale;
  return tc::launch_gemm_w8a8(g, st) == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}
