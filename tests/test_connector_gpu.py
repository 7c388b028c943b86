"""The embeddings connector on the GPU (src/ltx25-connector.cc) against the numpy
restatement of Ltx25Connector::forward: padded positions replaced by the
tiled registers, full attention, plain residuals, biased feed-forward, the
output norm.  The reference pads its golden deliberately (100 valid of 256,
tests/ltx25-connector-test.cc:13-14); so does the real-width case here.

Bars: the block's, on the output (6e-3 at one block's depth, 1e-2 here for
up to two) and on the connector's own contribution (output minus input,
3e-2), against an oracle on the same dequantized weights."""
import numpy as np
import pytest

from oracle import connector_np, lib

from test_block_gpu import bf16r, dev_bf16, host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("heads,hd,layers,regs,T,n_valid,norm_out,gated", [
    (4, 64, 2, 8, 32, 13, True, True),
    (2, 128, 2, 16, 48, 48, False, False),
    (32, 128, 1, 128, 256, 100, True, True),
])
def test_connector_matches_oracle(ctx, heads, hd, layers, regs, T, n_valid, norm_out, gated):
    import torch
    import ltx25_b200 as L
    dim = heads * hd
    t = connector_np.random_tensors(dim, heads, layers, regs, seed=heads + layers, gated=gated)
    c = L.Connector(ctx, heads, hd, layers, regs, norm_output=norm_out)
    deq = c.load(t)
    ow = {}
    for k, v in deq.items():
        ow[k] = bf16r(v) if (k.endswith(".bias") or "to_gate_logits" in k or
                             k == "learnable_registers") else v
    c.finalize()
    c.reserve(T)
    rng = np.random.default_rng(T)
    x = bf16r(rng.standard_normal((T, dim)))
    got = c.forward(dev_bf16(x), n_valid)
    torch.cuda.synchronize()
    ctx.check()
    want = connector_np.forward(ow, x, n_valid, heads, hd, layers, regs, norm_out)
    g = host(got)
    out_r = lib.rel_l2(g, want)
    print((heads, hd, layers, regs, T, n_valid), out_r)
    assert out_r < 1e-2, out_r
    if not norm_out:
        x0 = x.copy()
        if regs:
            for i in range(n_valid, T):
                x0[i] = ow["learnable_registers"].reshape(regs, dim)[i % regs]
        delta_r = lib.rel_l2(g - x0, want - x0)
        print("delta", delta_r)
        assert delta_r < 3e-2, delta_r
    # the registers are used: all-valid differs (tests/ltx25-connector-test.cc:135-142)
    if regs and n_valid < T:
        allv = c.forward(dev_bf16(x), T)
        torch.cuda.synchronize()
        assert lib.rel_l2(host(allv), g) > 1e-3
    # in place is the same
    xd = dev_bf16(x)
    c.forward(xd, n_valid, out=xd)
    torch.cuda.synchronize()
    assert torch.equal(xd, got)
    c.close()


def test_connector_refuses_bad_lengths(ctx):
    import ltx25_b200 as L
    t = connector_np.random_tensors(256, 4, 1, 8, seed=1)
    c = L.Connector(ctx, 4, 64, 1, 8)
    c.load(t)
    c.finalize()
    with pytest.raises(L.LtxError) as e:
        c.reserve(30)                  # not a multiple of the register count
    assert e.value.code == -2
    c.close()
    c = L.Connector(ctx, 4, 64, 1, 8)
    with pytest.raises(L.LtxError) as e:
        c.finalize()                   # nothing staged
    assert e.value.code == -7
    c.close()
