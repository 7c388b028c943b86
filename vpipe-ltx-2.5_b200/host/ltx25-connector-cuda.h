// ltx25-connector-cuda.h -- the embeddings connector on the GPU: the stack
// of 1-D transformer blocks between the text encoder and the DiT
// (Ltx25Connector, src/ltx25-connector.cc:38-260).  Per block: RMSNorm (no
// gain), q / k / v with bias, q / k RMS gain over the whole width and the
// 1-D index RoPE at the connector's own max_pos, full attention (the
// learnable registers have replaced every padded position, so no mask),
// optional per-head gate, out projection with bias and a PLAIN residual;
// RMSNorm, the biased GELU feed-forward, a plain residual.  Optionally a
// final RMSNorm.  Built from the block's pieces: the tcgen05 GEMM (the
// residual adds through its gated-residual epilogue at gate 1), the q/k
// norm + rope kernel and the attention.
#pragma once

#include <map>
#include <string>
#include <vector>

#include "ltx25-cuda-ops.h"

namespace ltx25 {

class CudaConnector {
public:
  CudaConnector(CudaOps* ops, int heads, int head_dim, int layers, int registers,
                bool norm_output, double theta, int max_pos, bool rope_f64)
      : _ops(ops), _heads(heads), _hd(head_dim), _dim(heads * head_dim), _layers(layers),
        _regs(registers), _norm_out(norm_output), _theta(theta), _max_pos(max_pos),
        _rope_f64(rope_f64)
  {
  }
  ~CudaConnector();

  // Names under the connector's root ("transformer_1d_blocks.3.attn1.to_q
  // .weight", "learnable_registers", ...).  A linear arrives as a w8g64
  // pack, or as a 2-D float tensor (a dense linear, the reference's
  // bind_qlinear without scales); everything else as f32.
  bool set_qlinear(const std::string& name, const uint32_t* codes, const void* scales,
                   const void* biases, int sb_dtype, int N, int K, bool on_device,
                   std::string* err);
  bool set_tensor(const std::string& name, const float* data, int rows, int cols,
                  bool on_device, std::string* err);
  bool finalize(std::string* err);
  // Size the scratch and the RoPE tables for `tokens` (a multiple of the
  // register count, Ltx25Connector::reserve, src/ltx25-connector.cc:138-180).
  bool reserve(int tokens, std::string* err);
  // out[tokens][dim] = connector(in), the first n_valid rows real, the rest
  // replaced by the registers (in == out is allowed).
  bool forward(cudaStream_t s, const __nv_bfloat16* in, __nv_bfloat16* out, int tokens,
               int n_valid, std::string* err);
  int dim() const { return _dim; }

private:
  struct Layer {
    QWeight q, k, v, o, gate, ff_in, ff_out;
    __nv_bfloat16 *q_b = nullptr, *k_b = nullptr, *v_b = nullptr, *o_b = nullptr,
                  *gate_b = nullptr, *ff_in_b = nullptr, *ff_out_b = nullptr;
    float *q_norm = nullptr, *k_norm = nullptr;
  };
  struct Staged {
    bool quant = false;
    QWeight q;
    std::vector<float> host;
    int rows = 0, cols = 0;
  };
  bool linear_(const std::string& name, int N, int K, QWeight* out, std::string* err);
  bool vec_bf16_(const std::string& name, int n, bool required, __nv_bfloat16** out,
                 std::string* err);
  bool vec_f32_(const std::string& name, int n, float** out, std::string* err);

  CudaOps* _ops;
  int _heads, _hd, _dim, _layers, _regs;
  bool _norm_out;
  double _theta;
  int _max_pos;
  bool _rope_f64;
  std::map<std::string, Staged> _staged;
  std::vector<Layer> _L;
  __nv_bfloat16* _registers = nullptr;
  std::vector<void*> _owned;
  bool _final = false;
  // scratch
  int _tokens = 0;
  __nv_bfloat16 *_a = nullptr, *_q = nullptr, *_k = nullptr, *_v = nullptr, *_qn = nullptr,
                *_kn = nullptr, *_o = nullptr, *_glog = nullptr, *_ff = nullptr;
  float *_cos = nullptr, *_sin = nullptr;
  std::vector<void*> _scratch;
};

}  // namespace ltx25
