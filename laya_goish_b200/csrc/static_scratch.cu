// Allocation-free Matrix::apply.
//
// Some callers cannot allocate device memory: a host application that hands
// every byte of HBM to its own pool at start-up (a serving framework's
// caching allocator, for example) leaves nothing for a stray cudaMalloc to
// take, and a thread that must not stall cannot afford cudaMalloc/cudaFree,
// which may synchronise the whole device.  laya_matrix_apply_static serves
// them: they pass device buffers they already own for the inputs and the
// output, and the staging the tensor-core GEMM needs (the weight decoded to
// F16, the activations rounded to F16, an error word) lives in one fixed
// array inside this library instead of in fresh allocations.
//
// The array is a file-scope __device__ object: every GPU on which the
// library's module is loaded holds LAYA_STATIC_SCRATCH_BYTES of it until the
// process exits.  Under CUDA's lazy module loading (the default) the module,
// and with it the array, is created on a device at the first call's set-up.
// Host code never uses the symbol itself as a pointer: on the first call on
// each device, with that device current, cudaGetSymbolAddress gives the
// device address, which is cached per device and passed to the kernels.
#include <algorithm>
#include <mutex>

#include "dequant.cuh"
#include "engine.h"
#include "gemm.h"
#include "kernels.h"
#include "laya_cuda.h"

namespace {

// GGUF blocks of a [rows][cols] weight -> the F16 [rows][ld] GEMM operand in
// one pass (gguf::decode, src/gguf.rs:250-336, then round to nearest F16:
// the same bits as decoding to F32 and rounding afterwards), with the pad
// columns cols..ld-1 set to zero.
__global__ void static_w16_kernel(int kind, const uint8_t* __restrict__ b, size_t nblocks, int rows, int cols,
                                  int ld, half* __restrict__ y) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < nblocks) laya::decode_raw_block(kind, b, i, laya::F16PadSink{y, cols, ld});
  const int pad = ld - cols;
  if (i < (size_t)rows * pad) y[(i / pad) * ld + cols + i % pad] = __float2half_rn(0.f);
}

constexpr size_t kScratchBytes = LAYA_STATIC_SCRATCH_BYTES;
__device__ __align__(256) unsigned char g_static_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of this device's copy of the scratch array (set-up on the
// first call per device).
int scratch_address(int dev, unsigned char** out) {
  if (dev < 0 || dev >= kMaxDevices) return laya::fail(LAYA_E_INVALID, "device index out of range");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p) return laya::cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
    g_scratch_addr[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_addr[dev]);
  return 0;
}

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

}  // namespace

extern "C" int laya_matrix_apply_static(uint32_t kind, const uint8_t* w, int rows, int cols, const float* x, int m,
                                        const float* bias, float* out, void* stream) {
  using namespace laya;
  int block, size;
  if (!ggml_layout(kind, &block, &size)) return fail(LAYA_E_INVALID, "unsupported GGML tensor type");
  if (!w || !x || !out || rows < 1 || cols < 1 || m < 0 || cols % block)
    return fail(LAYA_E_INVALID, "invalid matrix arguments");
  if (m == 0) return 0;
  const int ld = (cols + 7) / 8 * 8;
  // scratch layout: [error word | W F16 padded | x F16 padded]
  const size_t off_w16 = 256;
  const size_t off_x16 = off_w16 + align256((size_t)rows * ld * 2);
  const size_t need = off_x16 + align256((size_t)m * ld * 2);
  if (need > kScratchBytes)
    return fail(LAYA_E_INVALID, "matrix too large for the static scratch: needs " + std::to_string(need) +
                                    " bytes, limit " + std::to_string(kScratchBytes));
  int dev = 0;
  LAYA_CK(cudaGetDevice(&dev));
  int major = 0, sms = 0;
  LAYA_CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  LAYA_CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  if (major != 10) return fail(LAYA_E_CUDA, "not an sm_100 GPU");
  unsigned char* scratch = nullptr;
  if (int rc = scratch_address(dev, &scratch)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned* err = reinterpret_cast<unsigned*>(scratch);
  half* w16 = reinterpret_cast<half*>(scratch + off_w16);
  half* x16 = reinterpret_cast<half*>(scratch + off_x16);
  // The error word is the only scratch that must start at zero; everything
  // else is fully rewritten before it is read.
  LAYA_CK(cudaMemsetAsync(err, 0, 4, st));
  const size_t wbytes = (size_t)rows * cols / block * size;
  const size_t nblocks = wbytes / size, work = std::max(nblocks, (size_t)rows * (ld - cols));
  static_w16_kernel<<<(unsigned)((work + 255) / 256), 256, 0, st>>>((int)kind, w, nblocks, rows, cols, ld, w16);
  LAYA_CK(cudaGetLastError());
  LAYA_CK(f32_to_f16_pad(x, m, cols, ld, x16, st));
  GemmArgs a{};
  a.M = m;
  a.N = rows;
  a.K = cols;
  a.bias = bias;
  a.out = out;
  a.ldo = rows;
  a.err = err;
  a.budget = 4000000000ll;
  LAYA_CK(gemm_launch(EPI_F32, x16, ld, w16, ld, a, sms, st));
  unsigned h_err = 0;
  LAYA_CK(cudaMemcpyAsync(&h_err, err, 4, cudaMemcpyDeviceToHost, st));
  LAYA_CK(cudaStreamSynchronize(st));
  if (h_err) return fail(LAYA_E_TIMEOUT, "a device-side wait ran out of its budget");
  return 0;
}
