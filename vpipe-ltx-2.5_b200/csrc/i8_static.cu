// i8_static.cu -- a fixed device array for the int8 tier's activation scratch.
//
// ltx_qlinear_i8_static runs the int8 tier (per-token int8 activation codes,
// then the kind::i8 GEMM) with its scratch -- the codes and the per-token
// scales -- in the array below instead of in memory the context allocates.
// It serves callers that may not allocate device memory during a call: a
// runtime that owns every byte of HBM through its own pool and forbids
// cudaMalloc between its planning and execution phases, or code running
// where an allocation would synchronize the device at a bad moment.
//
// The array is a module global: every GPU that loads this library holds it
// (LTX_I8_STATIC_MAX_CODES + 4 * LTX_I8_STATIC_MAX_ROWS bytes) until the
// process exits.  All calls on a device share it and it keeps what the last
// call wrote; nothing in it needs clearing, because each call writes every
// code and scale its GEMM reads (the GEMM's tensor map stops at row M, and
// rows past it read as zero).  Two calls whose kernels overlap on the GPU
// (different streams, no ordering between them) race on it.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "../../include/ltx25_cuda.h"
#include "kernels.h"

namespace ltx {

namespace {

constexpr size_t kCodes = (size_t)LTX_I8_STATIC_MAX_CODES;
constexpr size_t kRows = (size_t)LTX_I8_STATIC_MAX_ROWS;
static_assert(kCodes % 256 == 0, "scales must start 256-byte aligned");

// [codes: kCodes int8][scales: kRows f32]
static __device__ __align__(256) unsigned char g_i8_static[kCodes + kRows * sizeof(float)];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

}  // namespace

// The device address of the array on `device`.  Looked up once per device,
// with that device current (the name g_i8_static is only a host-side handle
// in this file, not a device address); later calls read the cached pointer,
// which a device reset would leave stale (the header says so).
bool i8_static_scratch(int device, int8_t** codes, float** scales, std::string* err)
{
  if (device < 0 || device >= kMaxDevices) {
    if (err) *err = "i8_static: device ordinal out of range";
    return false;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_addr[device] == nullptr) {
    int cur = -1;
    cudaError_t e = cudaGetDevice(&cur);
    if (e == cudaSuccess && cur != device) e = cudaSetDevice(device);
    void* p = nullptr;
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&p, g_i8_static);
    if (cur >= 0 && cur != device) {
      const cudaError_t r = cudaSetDevice(cur);
      if (e == cudaSuccess) e = r;
    }
    if (e != cudaSuccess || p == nullptr) {
      if (err)
        *err = std::string("i8_static: cudaGetSymbolAddress: ") +
               cudaGetErrorString(e == cudaSuccess ? cudaErrorInvalidSymbol : e);
      return false;
    }
    g_addr[device] = p;
  }
  unsigned char* base = static_cast<unsigned char*>(g_addr[device]);
  *codes = reinterpret_cast<int8_t*>(base);
  *scales = reinterpret_cast<float*>(base + kCodes);
  return true;
}

}  // namespace ltx
