// tma_ingest.cu -- how many bytes a second one SM takes in through each
// load path the GEMMs could use, with no consumer work: a ring of 8 stages,
// each holding one k-block of the small-M w8g64 GEMM's operands (the
// activation box, 64 bf16 x 128 rows, SWIZZLE_128B; the code box, 64 u8 x
// 128 rows, SWIZZLE_64B; the 128 scale/zero-point words) or a subset, the
// activation rows alternatively copied by 128 threads with cp.async.  Run
// with 1, 16 and 148 CTAs (one per SM); prints cycles per stage and bytes
// per clock per SM.  A measurement tool for the GEMMs' roofline, built by
// vpipe-ltx-2.5_b200/build.py into lib/diag_tma_ingest; not part of the
// library.
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <cuda.h>
#include <cuda_runtime.h>
#include "../csrc/ptx.cuh"
using namespace ltx;
typedef CUresult (*PFN_enc)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                            const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                            CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                            CUtensorMapFloatOOBfill);
static PFN_enc enc;
static bool mk(CUtensorMap* m, CUtensorMapDataType dt, void* p, uint64_t inner, uint64_t outer,
               uint64_t rowb, uint32_t bi, uint32_t bo, CUtensorMapSwizzle sw)
{
  cuuint64_t d[2] = {inner, outer}, st[1] = {rowb};
  cuuint32_t b[2] = {bi, bo}, e[2] = {1, 1};
  return enc(m, dt, 2, p, d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
constexpr int S = 8;
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src)
{
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar)
{
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// mode 0: X + W(64B rows) + sz ; 1: X only ; 2: W only ; 3: X + W as 128B x 64 rows + sz
// mode 0: X + W(64B rows) + sz ; 1: X only ; 2: W only ; 3: X + W as 128B x 64 rows + sz
// mode 4: X by cp.async (128 threads) + W + sz by TMA ; 5: X by cp.async only
__global__ void __launch_bounds__(128, 1) k(const __grid_constant__ CUtensorMap tx,
                                            const __grid_constant__ CUtensorMap tw,
                                            const __grid_constant__ CUtensorMap tw2,
                                            const __grid_constant__ CUtensorMap tsz, int mode,
                                            int iters, int kblocks, const uint8_t* xg, int K,
                                            unsigned long long* out)
{
  extern __shared__ uint8_t raw[];
  uint8_t* base = (uint8_t*)(((uintptr_t)raw + 1023) & ~(uintptr_t)1023);
  __shared__ uint64_t bar[S];
  const bool lsu = mode >= 4;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) mbar_init(&bar[i], lsu ? 129 : 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (!lsu && threadIdx.x != 0) return;
  const int nt = blockIdx.x;
  unsigned long long t0 = 0;
  volatile int no_abort = 0;
  for (int it = 0; it < iters + S; ++it) {
    const int s = it % S;
    if (it >= S) {
      mbar_wait(&bar[s], ((it / S) - 1) & 1, &no_abort, nullptr, 0);
      if (it == S) t0 = clock64();
    }
    if (it >= iters) continue;
    const int kb = (it + nt * 3) % kblocks;
    uint8_t* sx = base + s * 16384;
    uint8_t* sw = base + S * 16384 + s * 8192;
    uint8_t* ss = base + S * (16384 + 8192) + s * 512;
    if (lsu) {
      // 128 rows x 128 B of X: thread t copies row t's 8 chunks
      const int r = threadIdx.x;
      if (r < 126) {
        const uint8_t* src = xg + ((size_t)r * K + kb * 64) * 2;
#pragma unroll
        for (int c = 0; c < 8; ++c) cp_async16(smem_u32(sx + r * 128 + 16 * (c ^ (r & 7))), src + 16 * c);
      }
      cp_async_arrive_noinc(&bar[s]);
      if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar[s], mode == 4 ? 8192 + 512 : 0);
        if (mode == 4) {
          tma_load_2d(&tw, &bar[s], sw, kb * 64, nt * 128);
          tma_load_2d(&tsz, &bar[s], ss, nt * 128, kb);
        }
      }
      continue;
    }
    uint32_t bytes = 0;
    if (mode == 0 || mode == 1 || mode == 3) bytes += 16384;
    if (mode == 0 || mode == 2 || mode == 3) bytes += 8192 + (mode == 2 ? 0 : 512);
    mbar_arrive_expect_tx(&bar[s], bytes);
    if (mode == 0 || mode == 1 || mode == 3) tma_load_2d(&tx, &bar[s], sx, kb * 64, 0);
    if (mode == 0 || mode == 2) tma_load_2d(&tw, &bar[s], sw, kb * 64, nt * 128);
    if (mode == 3) tma_load_2d(&tw2, &bar[s], sw, 0, (nt * kblocks + kb) * 64);
    if (mode == 0 || mode == 3) tma_load_2d(&tsz, &bar[s], ss, nt * 128, kb);
  }
  const unsigned long long t1 = clock64();
  if (threadIdx.x == 0) out[blockIdx.x] = t1 - t0;
}
int main()
{
  void* fn; cudaDriverEntryPointQueryResult q;
  cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  enc = (PFN_enc)fn;
  const int M = 126, K = 8192, N = 148 * 128, kbs = K / 64;
  void *x, *w, *sz; unsigned long long* out;
  cudaMalloc(&x, (size_t)M * K * 2); cudaMalloc(&w, (size_t)N * K); cudaMalloc(&sz, (size_t)N * (K / 64) * 4);
  cudaMalloc(&out, 148 * 8);
  cudaMemset(x, 0, (size_t)M * K * 2); cudaMemset(w, 0, (size_t)N * K); cudaMemset(sz, 0, (size_t)N * (K / 64) * 4);
  CUtensorMap tx, tw, tw2, tsz;
  bool ok = mk(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, K, M, (uint64_t)K * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) &&
            mk(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, K, N, K, 64, 128, CU_TENSOR_MAP_SWIZZLE_64B) &&
            mk(&tw2, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, 128, (uint64_t)N * K / 128, 128, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B) &&
            mk(&tsz, CU_TENSOR_MAP_DATA_TYPE_UINT32, sz, N, K / 64, (uint64_t)N * 4, 128, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!ok) { printf("encode failed\n"); return 1; }
  const int smem = 1024 + S * (16384 + 8192 + 512);
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const char* names[6] = {"X+W(64B rows)+sz", "X only", "W(64B rows) only", "X+W(128B rows)+sz",
                          "X cp.async + W,sz TMA", "X cp.async only"};
  for (int ctas : {1, 16, 148}) {
    for (int mode = 0; mode < 6; ++mode) {
      const int iters = 512;
      unsigned long long h[148];
      for (int rep = 0; rep < 3; ++rep) {
        k<<<ctas, 128, smem>>>(tx, tw, tw2, tsz, mode, iters, kbs, (const uint8_t*)x, K, out);
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) { printf("err %s\n", cudaGetErrorString(e)); return 1; }
      }
      cudaMemcpy(h, out, ctas * 8, cudaMemcpyDeviceToHost);
      double mean = 0; for (int i = 0; i < ctas; ++i) mean += h[i]; mean /= ctas;
      const int bytes = (mode == 1 || mode == 5 ? 16384 : mode == 2 ? 8192 : 16384 + 8192 + 512);
      const double per = mean / (iters - S);
      printf("ctas %3d %-20s %7.1f cycles/stage  %6.1f B/clk/SM\n", ctas, names[mode], per, bytes / per);
    }
  }
  return 0;
}
