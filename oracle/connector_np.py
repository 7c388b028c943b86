"""The embeddings connector restated in numpy (TEST INFRASTRUCTURE ONLY).

Ltx25Connector::forward (src/ltx25-connector.cc:182-260): the padded
positions (t >= n_valid) replaced by the learnable registers tiled over the
sequence (ltx_fill_registers, src/ltx25-kernels.metal:382-396); per block
RMSNorm, the attention of block_np.attention (whole-width q / k RMS gain,
the 1-D index RoPE at max_pos, full attention, per-head gate, biased out
projection) with a PLAIN residual, RMSNorm, the biased GELU feed-forward
with a plain residual; an optional final RMSNorm.  The reference's connector
goldens (conn_*_in / _out) are not in the tree: parity is to this
restatement of its code.
"""
import numpy as np

from . import block_np, rope_np

F32 = np.float32
EPS = 1e-6


def forward(t, x, n_valid, heads, head_dim, layers, registers, norm_output, max_pos=4096):
    x = np.asarray(x, F32).copy()
    T, dim = x.shape
    if registers > 0:
        regs = np.asarray(t["learnable_registers"], F32).reshape(registers, dim)
        for i in range(n_valid, T):
            x[i] = regs[i % registers]
    pe = rope_np.build_index_rope(T, max_pos, dim, heads)
    for i in range(layers):
        p = f"transformer_1d_blocks.{i}."
        a = block_np.rms_norm(x, EPS)
        att = block_np.attention(block_np._attn_params(t, p + "attn1"), a, a, pe, pe, heads,
                                 head_dim)
        x = (x + att).astype(F32)
        a = block_np.rms_norm(x, EPS)
        h = block_np.gelu_tanh(block_np.linear(a, t[p + "ff.net.0.proj.weight"],
                                               t[p + "ff.net.0.proj.bias"]))
        x = (x + block_np.linear(h, t[p + "ff.net.2.weight"], t[p + "ff.net.2.bias"])).astype(F32)
    if norm_output:
        x = block_np.rms_norm(x, EPS)
    return x


def random_tensors(dim, heads, layers, registers, seed=0, gated=True):
    rng = np.random.default_rng(seed)
    n = lambda *s, sc=0.02: (rng.standard_normal(s) * sc).astype(F32)
    t = {}
    if registers > 0:
        t["learnable_registers"] = n(registers, dim, sc=1.0)
    for i in range(layers):
        p = f"transformer_1d_blocks.{i}."
        for m in ("to_q", "to_k", "to_v", "to_out.0"):
            t[p + f"attn1.{m}.weight"] = n(dim, dim, sc=1.0 / np.sqrt(dim))
            t[p + f"attn1.{m}.bias"] = n(dim)
        t[p + "attn1.q_norm.weight"] = (1.0 + n(dim, sc=0.1)).astype(F32)
        t[p + "attn1.k_norm.weight"] = (1.0 + n(dim, sc=0.1)).astype(F32)
        if gated:
            t[p + "attn1.to_gate_logits.weight"] = n(heads, dim, sc=1.0 / np.sqrt(dim))
            t[p + "attn1.to_gate_logits.bias"] = n(heads)
        t[p + "ff.net.0.proj.weight"] = n(4 * dim, dim, sc=1.0 / np.sqrt(dim))
        t[p + "ff.net.0.proj.bias"] = n(4 * dim)
        t[p + "ff.net.2.weight"] = n(dim, 4 * dim, sc=1.0 / np.sqrt(4 * dim))
        t[p + "ff.net.2.bias"] = n(dim)
    return t
