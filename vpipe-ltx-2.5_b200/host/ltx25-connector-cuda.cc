// ltx25-connector-cuda.cc -- see ltx25-connector-cuda.h.
#include "ltx25-connector-cuda.h"

#include <cstring>

#include "../../include/ltx25_cuda.h"
#include "../csrc/block_ops.h"
#include "../csrc/kernels.h"

namespace ltx25 {

namespace {

bool fail(std::string* err, const std::string& m)
{
  if (err != nullptr) *err = m;
  return false;
}

bool ok_cuda(cudaError_t e, const char* what, std::string* err)
{
  if (e == cudaSuccess) return true;
  return fail(err, std::string(what) + ": " + cudaGetErrorString(e));
}

constexpr float kEps = 1e-6f;

}  // namespace

CudaConnector::~CudaConnector()
{
  for (auto& kv : _staged)
    if (kv.second.quant) free_qweight(&kv.second.q);
  for (Layer& l : _L)
    for (QWeight* w : {&l.q, &l.k, &l.v, &l.o, &l.gate, &l.ff_in, &l.ff_out}) free_qweight(w);
  for (void* p : _owned) cudaFree(p);
  for (void* p : _scratch) cudaFree(p);
}

bool CudaConnector::set_qlinear(const std::string& name, const uint32_t* codes,
                                const void* scales, const void* biases, int sb_dtype, int N,
                                int K, bool on_device, std::string* err)
{
  if (_final) return fail(err, "connector already finalized");
  Staged st;
  st.quant = true;
  if (!upload_qweight(*_ops, codes, scales, biases, sb_dtype, N, K, 8, 64, on_device, &st.q,
                      err))
    return false;
  st.rows = N;
  st.cols = K;
  auto it = _staged.find(name);
  if (it != _staged.end() && it->second.quant) free_qweight(&it->second.q);
  _staged[name] = std::move(st);
  return true;
}

bool CudaConnector::set_tensor(const std::string& name, const float* data, int rows, int cols,
                               bool on_device, std::string* err)
{
  if (_final) return fail(err, "connector already finalized");
  if (data == nullptr || rows <= 0) return fail(err, "set_tensor: null or empty " + name);
  Staged st;
  st.rows = rows;
  st.cols = cols > 0 ? cols : 1;
  const size_t n = (size_t)st.rows * st.cols;
  st.host.resize(n);
  if (on_device) {
    if (!ok_cuda(cudaMemcpy(st.host.data(), data, n * 4, cudaMemcpyDeviceToHost), "stage",
                 err))
      return false;
  } else {
    std::memcpy(st.host.data(), data, n * 4);
  }
  auto it = _staged.find(name);
  if (it != _staged.end() && it->second.quant) free_qweight(&it->second.q);
  _staged[name] = std::move(st);
  return true;
}

bool CudaConnector::linear_(const std::string& name, int N, int K, QWeight* out,
                            std::string* err)
{
  auto it = _staged.find(name);
  if (it == _staged.end()) return fail(err, "missing tensor '" + name + "'");
  Staged& st = it->second;
  if (st.rows != N || st.cols != K)
    return fail(err, "tensor '" + name + "' is [" + std::to_string(st.rows) + "][" +
                         std::to_string(st.cols) + "], want [" + std::to_string(N) + "][" +
                         std::to_string(K) + "] (shape)");
  if (st.quant) {
    *out = st.q;
    st.q = QWeight{};
    st.quant = false;
    return true;
  }
  // a dense linear: bf16 of the staged f32 (round to nearest even)
  std::vector<uint16_t> h(st.host.size());
  for (size_t i = 0; i < h.size(); ++i) {
    uint32_t u;
    std::memcpy(&u, &st.host[i], 4);
    h[i] = (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
  }
  return upload_dweight(*_ops, h.data(), N, K, false, out, err);
}

bool CudaConnector::vec_bf16_(const std::string& name, int n, bool required,
                              __nv_bfloat16** out, std::string* err)
{
  *out = nullptr;
  auto it = _staged.find(name);
  if (it == _staged.end()) return required ? fail(err, "missing tensor '" + name + "'") : true;
  if (it->second.quant || it->second.host.size() != (size_t)n)
    return fail(err, "tensor '" + name + "' has " + std::to_string(it->second.host.size()) +
                         " elements, want " + std::to_string(n) + " (shape)");
  std::vector<uint16_t> h((size_t)n);
  for (int i = 0; i < n; ++i) {
    uint32_t u;
    std::memcpy(&u, &it->second.host[(size_t)i], 4);
    h[(size_t)i] = (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
  }
  void* d = nullptr;
  if (!ok_cuda(cudaMalloc(&d, (size_t)n * 2), "cudaMalloc(connector)", err)) return false;
  _owned.push_back(d);
  if (!ok_cuda(cudaMemcpy(d, h.data(), (size_t)n * 2, cudaMemcpyHostToDevice), "upload", err))
    return false;
  *out = static_cast<__nv_bfloat16*>(d);
  return true;
}

bool CudaConnector::vec_f32_(const std::string& name, int n, float** out, std::string* err)
{
  *out = nullptr;
  auto it = _staged.find(name);
  if (it == _staged.end()) return fail(err, "missing tensor '" + name + "'");
  if (it->second.quant || it->second.host.size() != (size_t)n)
    return fail(err, "tensor '" + name + "' has the wrong size (shape)");
  void* d = nullptr;
  if (!ok_cuda(cudaMalloc(&d, (size_t)n * 4), "cudaMalloc(connector)", err)) return false;
  _owned.push_back(d);
  if (!ok_cuda(cudaMemcpy(d, it->second.host.data(), (size_t)n * 4, cudaMemcpyHostToDevice),
               "upload", err))
    return false;
  *out = static_cast<float*>(d);
  return true;
}

bool CudaConnector::finalize(std::string* err)
{
  if (_final) return true;
  if (_dim % 64 != 0 || _layers <= 0) return fail(err, "connector shape: width % 64, layers");
  const int d = _dim, h = 4 * _dim;   // the feed-forward is 4x (src/ltx25-connector.cc:51-53)
  if (_regs > 0 && !vec_bf16_("learnable_registers", _regs * d, true, &_registers, err))
    return false;
  _L.resize((size_t)_layers);
  for (int i = 0; i < _layers; ++i) {
    Layer& l = _L[(size_t)i];
    const std::string p = "transformer_1d_blocks." + std::to_string(i) + ".";
    if (!linear_(p + "attn1.to_q.weight", d, d, &l.q, err) ||
        !linear_(p + "attn1.to_k.weight", d, d, &l.k, err) ||
        !linear_(p + "attn1.to_v.weight", d, d, &l.v, err) ||
        !linear_(p + "attn1.to_out.0.weight", d, d, &l.o, err) ||
        !linear_(p + "ff.net.0.proj.weight", h, d, &l.ff_in, err) ||
        !linear_(p + "ff.net.2.weight", d, h, &l.ff_out, err) ||
        !vec_bf16_(p + "attn1.to_q.bias", d, true, &l.q_b, err) ||
        !vec_bf16_(p + "attn1.to_k.bias", d, true, &l.k_b, err) ||
        !vec_bf16_(p + "attn1.to_v.bias", d, true, &l.v_b, err) ||
        !vec_bf16_(p + "attn1.to_out.0.bias", d, true, &l.o_b, err) ||
        // the connector's feed-forward has its biases (src/ltx25-connector.cc:101-106)
        !vec_bf16_(p + "ff.net.0.proj.bias", h, true, &l.ff_in_b, err) ||
        !vec_bf16_(p + "ff.net.2.bias", d, true, &l.ff_out_b, err) ||
        !vec_f32_(p + "attn1.q_norm.weight", d, &l.q_norm, err) ||
        !vec_f32_(p + "attn1.k_norm.weight", d, &l.k_norm, err))
      return false;
    if (_staged.count(p + "attn1.to_gate_logits.weight")) {
      if (!linear_(p + "attn1.to_gate_logits.weight", _heads, d, &l.gate, err) ||
          !vec_bf16_(p + "attn1.to_gate_logits.bias", _heads, false, &l.gate_b, err))
        return false;
    }
  }
  for (auto& kv : _staged)
    if (kv.second.quant) free_qweight(&kv.second.q);
  _staged.clear();
  _final = true;
  return true;
}

bool CudaConnector::reserve(int tokens, std::string* err)
{
  if (!_final) return fail(err, "reserve before finalize");
  if (tokens <= 0) return fail(err, "connector shape: tokens must be positive");
  if (_regs > 0 && tokens % _regs != 0)
    return fail(err, "connector shape: sequence length " + std::to_string(tokens) +
                         " is not a multiple of the register count " + std::to_string(_regs));
  if (tokens == _tokens) return true;
  for (void* p : _scratch) cudaFree(p);
  _scratch.clear();
  const size_t T = (size_t)tokens, d = (size_t)_dim;
  auto get = [&](size_t elems, size_t es, void** p) {
    if (!ok_cuda(cudaMalloc(p, elems * es + 256), "cudaMalloc(connector scratch)", err))
      return false;
    _scratch.push_back(*p);
    return true;
  };
  if (!get(T * d, 2, (void**)&_a) || !get(T * d, 2, (void**)&_q) ||
      !get(T * d, 2, (void**)&_k) || !get(T * d, 2, (void**)&_v) ||
      !get(T * d, 2, (void**)&_qn) || !get(T * d, 2, (void**)&_kn) ||
      !get(T * d, 2, (void**)&_o) || !get(T * (size_t)_heads, 2, (void**)&_glog) ||
      !get(T * 4 * d, 2, (void**)&_ff))
    return false;
  // The 1-D index RoPE at the connector's own max_pos: position i spans
  // [i, i + 1) (build_index_rope, src/ltx25-rope.cc:266-279).
  std::vector<double> st(T), en(T);
  for (size_t i = 0; i < T; ++i) {
    st[i] = (double)i;
    en[i] = (double)i + 1.0;
  }
  const size_t tab = (size_t)_heads * T * (size_t)(_hd / 2);
  std::vector<float> c(tab), s(tab);
  if (ltx_rope_table(st.data(), en.data(), 1, tokens, &_max_pos, _dim, _heads, _theta,
                     _rope_f64 ? 1 : 0, c.data(), s.data()) != LTX_OK)
    return fail(err, "connector RoPE table failed");
  if (!get(tab, 4, (void**)&_cos) || !get(tab, 4, (void**)&_sin) ||
      !ok_cuda(cudaMemcpy(_cos, c.data(), tab * 4, cudaMemcpyHostToDevice), "rope", err) ||
      !ok_cuda(cudaMemcpy(_sin, s.data(), tab * 4, cudaMemcpyHostToDevice), "rope", err))
    return false;
  if (!_ops->reserve_attention(tokens, _dim, err)) return false;
  _tokens = tokens;
  return true;
}

bool CudaConnector::forward(cudaStream_t s, const __nv_bfloat16* in, __nv_bfloat16* out,
                            int tokens, int n_valid, std::string* err)
{
  if (!_final) return fail(err, "forward before finalize");
  if (tokens != _tokens)
    return fail(err, "connector: reserve() sized for " + std::to_string(_tokens) +
                         " tokens, forward wants " + std::to_string(tokens) + " (shape)");
  if (in == nullptr || out == nullptr) return fail(err, "connector: null in or out");
  if (n_valid < 0 || n_valid > tokens) return fail(err, "connector shape: n_valid");
  const int T = tokens, d = _dim, h = 4 * _dim;
  const float* one = _ops->ones(h, s, err);
  if (one == nullptr) return false;
  if (in != out &&
      !ok_cuda(cudaMemcpyAsync(out, in, (size_t)T * d * 2, cudaMemcpyDeviceToDevice, s),
               "connector copy", err))
    return false;
  if (_regs > 0 && ltx::launch_fill_registers(out, d, _registers, d, _regs, n_valid, T, s) != 0)
    return fail(err, "register fill launch failed");
  for (const Layer& l : _L) {
    // pre-norm + self-attention, plain residual (src/ltx25-connector.cc:212-248)
    if (ltx::launch_ada_zero(out, d, _a, d, T, d, nullptr, nullptr, kEps, true, s) != 0)
      return fail(err, "connector norm launch failed");
    if (!_ops->linear(s, _a, d, l.q, l.q_b, _q, d, T, d, d, ltx::EPI_STORE, nullptr, err) ||
        !_ops->linear(s, _a, d, l.k, l.k_b, _k, d, T, d, d, ltx::EPI_STORE, nullptr, err) ||
        !_ops->linear(s, _a, d, l.v, l.v_b, _v, d, T, d, d, ltx::EPI_STORE, nullptr, err))
      return false;
    if (ltx::launch_qk_norm_rope(_q, d, _qn, d, T, _heads, _hd, l.q_norm, _cos, _sin, kEps, s,
                                 nullptr, d, 0, T, 0) != 0 ||
        ltx::launch_qk_norm_rope(_k, d, _kn, d, T, _heads, _hd, l.k_norm, _cos, _sin, kEps, s,
                                 nullptr, d, 0, T, 0) != 0)
      return fail(err, "connector q/k norm + rope launch failed");
    const __nv_bfloat16* glog = nullptr;
    if (l.gate.N > 0) {
      if (!_ops->linear(s, _a, d, l.gate, l.gate_b, _glog, _heads, T, d, _heads,
                        ltx::EPI_STORE, nullptr, err))
        return false;
      glog = _glog;
    }
    if (!_ops->attention(s, _qn, d, _kn, d, _v, d, _o, d, glog, _heads, T, T, _heads, _hd, err,
                         -1))
      return false;
    if (!_ops->linear(s, _o, d, l.o, l.o_b, out, d, T, d, d, ltx::EPI_GATED_RES, one, err))
      return false;
    // pre-norm + feed-forward, plain residual
    if (ltx::launch_ada_zero(out, d, _a, d, T, d, nullptr, nullptr, kEps, true, s) != 0)
      return fail(err, "connector norm launch failed");
    if (!_ops->linear(s, _a, d, l.ff_in, l.ff_in_b, _ff, h, T, d, h, ltx::EPI_GELU, nullptr,
                      err) ||
        !_ops->linear(s, _ff, h, l.ff_out, l.ff_out_b, out, d, T, h, d, ltx::EPI_GATED_RES, one,
                      err))
      return false;
  }
  if (_norm_out && ltx::launch_ada_zero(out, d, out, d, T, d, nullptr, nullptr, kEps, true, s) != 0)
    return fail(err, "connector output norm launch failed");
  return true;
}

}  // namespace ltx25
