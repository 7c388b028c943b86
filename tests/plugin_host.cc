// plugin_host.cc -- a stand-in vpipe host for the plugin tests.  It loads
// lib/vpipe-ltx-2.5-b200.so the way a host loads a plugin (dlopen, the ABI
// integer and the info record first, then the registration entry with the
// host's context), checks what the plugin requires and registers, and then
// drives the family's linear through the registered kernel table:
//
//   plugin_host <plugin.so> cpu   no GPU: the table's entries reach the C ABI
//                                 and report its errors
//   plugin_host <plugin.so> gpu   one w8g64 linear on device 0 against a
//                                 dequantise-then-dense f64 product on the host
//
// Built by tests/test_plugin_cpu.py and tests/test_plugin_gpu.py with
// -Wall -Wextra -Werror against the in-repo stub headers.
#include <dlfcn.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <random>
#include <string>
#include <vector>

#include "plugin/plugin-abi.h"
#include "plugin/plugin-context.h"
#include "ltx25_plugin.h"

#include <cuda_runtime.h>

namespace {

class RecordingContext : public vpipe::VpipePluginContext {
public:
  bool register_kernel_table(const vpipe::KernelTable& t) override
  {
    if (tables_.count(t.name) != 0) return false;   // first registration wins
    tables_[t.name] = t;
    return true;
  }
  const vpipe::KernelTable* find_kernel_table(const char* name) const override
  {
    auto it = tables_.find(name);
    return it == tables_.end() ? nullptr : &it->second;
  }
  size_t size() const { return tables_.size(); }

private:
  std::map<std::string, vpipe::KernelTable> tables_;
};

uint16_t bf16_rne(double v)
{
  float f = (float)v;                 // exact for the values built below
  uint32_t u;
  std::memcpy(&u, &f, 4);
  u += 0x7FFF + ((u >> 16) & 1);
  return (uint16_t)(u >> 16);
}

double bf16_val(uint16_t h)
{
  uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

int run_gpu(const ltx25_cuda_kernels* k)
{
  char err[512] = {0};
  ltx25_ops* ops = nullptr;
  int rc = k->ops_create(0, &ops, err, sizeof err);
  if (rc != LTX_OK) {
    std::printf("ops_create %d %s\n", rc, err);
    return 1;
  }
  const int M = 192, K = 512, N = 256, G = K / 64;
  std::mt19937 rng(7);
  std::uniform_int_distribution<int> code(0, 255);
  std::normal_distribution<float> nrm(0.f, 1.f);
  std::vector<uint32_t> codes((size_t)N * K / 4, 0);
  std::vector<uint16_t> sc((size_t)N * G), zp((size_t)N * G), xb((size_t)M * K);
  std::vector<uint8_t> q((size_t)N * K);
  for (size_t i = 0; i < q.size(); ++i) {
    q[i] = (uint8_t)code(rng);
    codes[i / 4] |= (uint32_t)q[i] << (8 * (i % 4));
  }
  for (size_t i = 0; i < sc.size(); ++i) {
    sc[i] = bf16_rne(0.0004 * (1.0 + 0.25 * std::fabs(nrm(rng))));
    zp[i] = bf16_rne(-0.05 * (1.0 + 0.1 * nrm(rng)));
  }
  for (auto& v : xb) v = bf16_rne(nrm(rng));
  ltx_qweight* w = nullptr;
  rc = k->bind_qlinear(ops, codes.data(), sc.data(), zp.data(), LTX_SB_BF16, N, K, &w, err,
                       sizeof err);
  if (rc != LTX_OK) {
    std::printf("bind_qlinear %d %s\n", rc, err);
    return 1;
  }
  void *dx = nullptr, *dy = nullptr;
  if (cudaMalloc(&dx, xb.size() * 2) != cudaSuccess ||
      cudaMalloc(&dy, (size_t)M * N * 2) != cudaSuccess) {
    std::printf("cudaMalloc failed\n");
    return 1;
  }
  cudaMemcpy(dx, xb.data(), xb.size() * 2, cudaMemcpyHostToDevice);
  rc = k->linear(ops, nullptr, dx, w, nullptr, dy, M, K, N, err, sizeof err);
  if (rc != LTX_OK) {
    std::printf("linear %d %s\n", rc, err);
    return 1;
  }
  rc = k->wait_ok(ops, nullptr, err, sizeof err);
  std::vector<uint16_t> y((size_t)M * N);
  cudaMemcpy(y.data(), dy, y.size() * 2, cudaMemcpyDeviceToHost);
  // dequantise-then-dense: w = bf16(s * q + z), one rounding; f64 sums
  double num = 0, den = 0;
  for (int n = 0; n < N; ++n) {
    std::vector<double> wr(K);
    for (int kk = 0; kk < K; ++kk) {
      const size_t g = (size_t)n * G + kk / 64;
      wr[kk] = bf16_val(bf16_rne(bf16_val(sc[g]) * q[(size_t)n * K + kk] + bf16_val(zp[g])));
    }
    for (int m = 0; m < M; ++m) {
      double acc = 0;
      for (int kk = 0; kk < K; ++kk) acc += bf16_val(xb[(size_t)m * K + kk]) * wr[kk];
      const double d = bf16_val(y[(size_t)m * N + n]) - acc;
      num += d * d;
      den += acc * acc;
    }
  }
  std::printf("gpu linear wait_ok %d rel_l2 %.3e\n", rc, std::sqrt(num / den));
  cudaFree(dx);
  cudaFree(dy);
  k->qweight_free(w);
  k->ops_destroy(ops);
  return 0;
}

}  // namespace

int main(int argc, char** argv)
{
  if (argc < 3) {
    std::fprintf(stderr, "usage: plugin_host <plugin.so> cpu|gpu\n");
    return 2;
  }
  void* so = dlopen(argv[1], RTLD_NOW | RTLD_LOCAL);
  if (so == nullptr) {
    std::printf("dlopen failed: %s\n", dlerror());
    return 1;
  }
  auto abi = reinterpret_cast<int (*)()>(dlsym(so, "vpipe_plugin_abi"));
  auto info = reinterpret_cast<const VpipePluginInfo* (*)()>(dlsym(so, "vpipe_plugin_info"));
  auto reg = reinterpret_cast<void (*)(vpipe::VpipePluginContext*)>(
      dlsym(so, "vpipe_plugin_register"));
  if (abi == nullptr || info == nullptr || reg == nullptr) {
    std::printf("missing plugin symbol\n");
    return 1;
  }
  const VpipePluginInfo* in = info();
  std::printf("abi %d schema %d name %s\n", abi(), in->schema, in->name);
  std::string req;
  for (const char* const* r = in->requires_features; r != nullptr && *r != nullptr; ++r)
    req += std::string(req.empty() ? "" : ",") + *r;
  std::printf("requires %s\n", req.c_str());
  RecordingContext host;
  reg(nullptr);                 // a null context is ignored, as in the reference
  reg(&host);
  const size_t n1 = host.size();
  reg(&host);                   // a second registration of the same name is refused
  std::printf("tables %zu %zu\n", n1, host.size());
  const vpipe::KernelTable* t = host.find_kernel_table(LTX25_CUDA_KERNELS_NAME);
  if (t == nullptr) {
    std::printf("no table %s\n", LTX25_CUDA_KERNELS_NAME);
    return 1;
  }
  const auto* k = static_cast<const ltx25_cuda_kernels*>(t->table);
  std::printf("table %s backend %s version %d abi %d size_ok %d\n", t->name, t->backend,
              k->version, k->abi, t->table_bytes == sizeof(ltx25_cuda_kernels) ? 1 : 0);
  if (std::strcmp(argv[2], "gpu") == 0) return run_gpu(k);

  char err[512] = {0};
  ltx25_ops* ops = nullptr;
  int rc = k->ops_create(9999, &ops, err, sizeof err);      // no such device anywhere
  std::printf("ops_create %d null %d msg %s\n", rc, ops == nullptr ? 1 : 0, err);
  rc = k->linear(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 1, 64, 64, err,
                 sizeof err);
  std::printf("linear_null %d\n", rc);
  std::printf("i8_takes %d\n", k->i8_takes(nullptr, 8160, 4096, 16384));
  ltx25_block* b = nullptr;
  rc = k->block_create(nullptr, 4096, 32, 2048, 32, &b, err, sizeof err);
  std::printf("block_create_null %d\n", rc);
  rc = k->block_finalize(nullptr, err, sizeof err);
  std::printf("block_finalize_null %d\n", rc);
  dlclose(so);
  return 0;
}
