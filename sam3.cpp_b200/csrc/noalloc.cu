// 3x3 convolution entry point that allocates no device memory.
//
// Some callers of this library cannot allocate device memory: a host that
// hands the library a fixed memory budget owned by another allocator (a
// game or video pipeline with a pre-sized pool), a plugin loaded into a
// process whose CUDA context is managed elsewhere and forbids cudaMalloc, or
// a real-time thread where cudaMalloc / cudaFree would synchronise the device
// and stall other streams. s3b_op_conv3x3 needs an im2col workspace (and a
// device error word) from its s3b_ctx, which allocates them with cudaMalloc.
// s3b_conv3x3_noalloc instead uses one file-scope __device__ array of fixed
// size for both: the library claims it when it is loaded, on every GPU that
// loads it, and keeps it until the process exits.
//
// Host code must not pass the array's name to a kernel: on the host it is a
// stand-in symbol, not a device address. The device address is looked up
// once per device with cudaGetSymbolAddress (with that device current) on
// the first call made on that device, so the first call on each device
// should come before any stream capture.
//
// All calls share the array and it keeps the previous call's contents: the
// error word is cleared at the start of every call; the im2col region is
// fully rewritten before it is read. The call only enqueues work, so a
// device-side failure (a bounded wait in the GEMM that timed out) cannot be
// in its return code: s3b_conv3x3_noalloc_status reads (and clears) the
// error word once the caller has waited for the stream. Calls whose work overlaps on the GPU
// (different streams, or different host threads without ordering) race on
// the array and must be serialised by the caller.
#include <stdio.h>

#include <mutex>

#include "../../include/sam3_b200.h"
#include "kernels.h"

namespace {

constexpr size_t kErrRegion = 256;  // error word of the GEMM's bounded waits (first 4 bytes)
__device__ __align__(256) unsigned char g_noalloc_scratch[kErrRegion + S3B_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_addr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (looked up once).
int scratch_address(int dev, unsigned char** out) {
  if (dev < 0 || dev >= kMaxDevices) return S3B_ERR_ARG;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      fprintf(stderr, "s3b_conv3x3_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", dev,
              cudaGetErrorString(e));
      return S3B_ERR_CUDA;
    }
    g_addr[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_addr[dev];
  return S3B_OK;
}

}  // namespace

extern "C" int s3b_conv3x3_noalloc(const void* x, int B, int H, int W, int C, const void* w, const float* bias,
                                   float* out, int Cout, void* stream) {
  if (!x || !w || !out || B <= 0 || H <= 0 || W <= 0 || C <= 0 || Cout <= 0 || C % 8 || Cout % 8) {
    fprintf(stderr, "s3b_conv3x3_noalloc: bad arguments\n");
    return S3B_ERR_ARG;
  }
  const unsigned long long M = (unsigned long long)B * H * W;
  const unsigned long long need = M * 9ull * (unsigned long long)C * 2ull;
  if (need > (unsigned long long)S3B_NOALLOC_SCRATCH_BYTES) {
    fprintf(stderr,
            "s3b_conv3x3_noalloc: B*H*W*9*C*2 = %llu bytes of im2col scratch exceeds the %llu-byte static "
            "scratch; use s3b_op_conv3x3 or split the batch\n",
            need, (unsigned long long)S3B_NOALLOC_SCRATCH_BYTES);
    return S3B_ERR_ARG;
  }
  if (M > 0x7fffffffull) return S3B_ERR_ARG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return S3B_ERR_CUDA;
  unsigned char* base = nullptr;
  int rc = scratch_address(dev, &base);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int* err = reinterpret_cast<int*>(base);
  __half* col = reinterpret_cast<__half*>(base + kErrRegion);
  if (cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess) return S3B_ERR_CUDA;
  if (s3b::im2col_3x3_cl(reinterpret_cast<const __half*>(x), B, H, W, C, col, st)) return S3B_ERR_CUDA;
  s3b::EpiParams ep;
  ep.mode = s3b::EPI_STORE;
  ep.bias = bias;
  ep.out = out;
  ep.out_f32 = 1;
  ep.ldo = Cout;
  rc = s3b::gemm_f16(col, 9LL * C, reinterpret_cast<const __half*>(w), 9LL * C, (int)M, Cout, 9 * C, ep, err, st);
  // launcher codes: -1..-11 argument / alignment checks (-11: a pointer or row stride not 16-byte
  // aligned, -10 no tensor-map encoder), below -11 CUDA errors
  if (rc == 0) return S3B_OK;
  if (rc == -10) return S3B_ERR_CUDA;
  return rc < -11 ? S3B_ERR_CUDA : S3B_ERR_ARG;
}

extern "C" int s3b_conv3x3_noalloc_status(int* code) {
  if (!code) return S3B_ERR_ARG;
  *code = 0;
  int h = 0;
  // the word is the first int of the scratch array on the current device (no allocation, no lookup)
  cudaError_t e = cudaMemcpyFromSymbol(&h, g_noalloc_scratch, sizeof(int), 0, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    fprintf(stderr, "s3b_conv3x3_noalloc_status: reading the error word failed: %s\n", cudaGetErrorString(e));
    return S3B_ERR_CUDA;
  }
  if (h == 0) return S3B_OK;
  *code = h;
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_noalloc_scratch, &zero, sizeof(int), 0, cudaMemcpyHostToDevice);
  fprintf(stderr, "s3b_conv3x3_noalloc: a bounded device wait timed out (code %d); the output is incomplete\n", h);
  return e == cudaSuccess ? S3B_ERR_DEVICE : S3B_ERR_CUDA;
}
