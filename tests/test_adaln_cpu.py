"""The trunk's adaLN chains on the host (src/ltx25-dit.cc:51-160):
the library's chain against the numpy restatement of Ltx25Dit::adaln_,
the [cos | sin] order and embedded_timestep's tap as controls, thread-count
independence, and the chain bound from a checkpoint."""
import numpy as np
import pytest

from oracle import adaln_np, lib

import st_file

DIM, OUT = 64, 9 * 64


def _weights(seed):
    rng = np.random.default_rng(seed)
    f = lambda *s, sc=1.0: lib.f32_to_bf16((rng.standard_normal(s) * sc).astype(np.float32))
    return (f(DIM, 256, sc=0.1), f(DIM, sc=0.1), f(DIM, DIM, sc=0.15), f(DIM, sc=0.1),
            f(OUT, DIM, sc=0.15), f(OUT, sc=0.1))


@pytest.mark.parametrize("t", [0.0, 1.0, 37.5, 500.0, 999.0])
def test_chain_matches_restatement(t):
    import ltx25_b200 as L
    w = _weights(1)
    a = L.AdaLN(*w)
    out, emb = a(t)
    want, want_emb = adaln_np.chain(t, *w)
    assert lib.rel_l2(out, want) < 1e-6
    assert lib.rel_l2(emb, want_emb) < 1e-6
    a.close()


@pytest.mark.parametrize("t", [0.0, 37.5, 999.0])
def test_chain_matches_the_reference_helpers(t):
    """The library's host chain against Ltx25Dit::adaln_'s own helpers
    (timestep_sinusoid_, gemv_host_, silu_; src/ltx25-dit.cc:30-160),
    compiled from the reference sources into oracle/_ref."""
    from oracle import ref
    if not ref.available():
        pytest.skip("oracle/_ref not built (no reference tree at build time)")
    import ltx25_b200 as L
    w = _weights(4)
    a = L.AdaLN(*w)
    out, emb = a(t)
    want, want_emb = ref.adaln_chain(t, *w)
    assert lib.rel_l2(out, want) < 1e-6
    assert lib.rel_l2(emb, want_emb) < 1e-6
    a.close()


def test_controls_and_threads():
    import ltx25_b200 as L
    w = _weights(2)
    a = L.AdaLN(*w)
    out, emb = a(250.0, threads=1)
    out8, emb8 = a(250.0, threads=8)
    assert np.array_equal(out, out8) and np.array_equal(emb, emb8)
    # [sin | cos] instead: a clean forward driven by the wrong half
    s = adaln_np.sinusoid(250.0)
    flipped = np.concatenate([s[128:], s[:128]])
    h1 = adaln_np.silu(adaln_np.gemv(flipped, w[0], w[1]))
    wrong = adaln_np.gemv(adaln_np.silu(adaln_np.gemv(h1, w[2], w[3])), w[4], w[5])
    assert lib.rel_l2(out, wrong) > 0.05
    # embedded_timestep is the SECOND linear's output, not the third's
    assert emb.shape == (DIM,)
    assert lib.rel_l2(emb, adaln_np.chain(250.0, *w)[1]) < 1e-6
    a.close()


def test_chain_from_checkpoint(tmp_path):
    import ltx25_b200 as L
    w = _weights(3)
    pre = "model.diffusion_model.adaln_single."
    names = ["emb.timestep_embedder.linear_1.weight", "emb.timestep_embedder.linear_1.bias",
             "emb.timestep_embedder.linear_2.weight", "emb.timestep_embedder.linear_2.bias",
             "linear.weight", "linear.bias"]
    tensors = {pre + n: a for n, a in zip(names, w)}
    # one tensor stored F32: the reader rounds it to bf16 as the loader does
    tensors[pre + "linear.weight"] = lib.bf16_to_f32(w[4])
    bf = tuple(pre + n for n in names if n != "linear.weight")
    p = st_file.write(tmp_path / "trunk.safetensors", tensors, bf16=bf)
    st = L.SafeTensors(p)
    a = L.AdaLN(st=st, prefix=pre)
    assert (a.dim, a.out_dim) == (DIM, OUT)
    out, emb = a(640.0)
    want, want_emb = adaln_np.chain(640.0, *w)
    assert lib.rel_l2(out, want) < 1e-6 and lib.rel_l2(emb, want_emb) < 1e-6
    with pytest.raises(L.LtxError) as e:
        L.AdaLN(st=st, prefix="model.diffusion_model.audio_adaln_single.")
    assert e.value.code == -7
    a.close()
    st.close()


_SCALAR = """
import sys, numpy as np
sys.path.insert(0, sys.argv[1])
import ltx25_b200 as L
w = [np.load(sys.argv[2] + f"/w{i}.npy") for i in range(6)]
out, emb = L.AdaLN(*w)(float(sys.argv[3]))
np.save(sys.argv[2] + "/out.npy", out)
np.save(sys.argv[2] + "/emb.npy", emb)
"""


@pytest.mark.parametrize("in_dim", [64, 67, 4096])
def test_vector_and_scalar_sums_are_bit_identical(tmp_path, in_dim):
    """The host's vector dot (AVX2 + FMA) and the scalar one sum the same
    eight partial sums in the same order, and f32 x bf16 products are exact
    in f64: the chain's bits must not depend on which one ran (the scalar
    form runs in a child process with LTX25_HOST_SIMD=0).  in_dim 67 leaves
    a tail after the last full group of eight."""
    import os
    import subprocess
    import sys
    import ltx25_b200 as L
    rng = np.random.default_rng(in_dim)
    f = lambda *s, sc=1.0: lib.f32_to_bf16((rng.standard_normal(s) * sc).astype(np.float32))
    w = (f(in_dim, 256, sc=0.1), f(in_dim, sc=0.1), f(in_dim, in_dim, sc=0.15),
         f(in_dim, sc=0.1), f(3 * in_dim, in_dim, sc=0.15), f(3 * in_dim, sc=0.1))
    for i, a in enumerate(w):
        np.save(tmp_path / f"w{i}.npy", a)
    out, emb = L.AdaLN(*w)(123.25)
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                       "vpipe-ltx-2.5_b200")
    env = dict(os.environ, LTX25_HOST_SIMD="0")
    subprocess.run([sys.executable, "-c", _SCALAR, pkg, str(tmp_path), "123.25"], env=env,
                   check=True, timeout=300)
    assert np.array_equal(out.view(np.uint32), np.load(tmp_path / "out.npy").view(np.uint32))
    assert np.array_equal(emb.view(np.uint32), np.load(tmp_path / "emb.npy").view(np.uint32))
    want, _ = adaln_np.chain(123.25, *w)
    assert lib.rel_l2(out, want) < 1e-6


def test_a_step_of_chains_at_once_equals_each_alone():
    """ltx_adaln_run_many (a denoise step's chains on one thread set, rows
    split across the chains) gives each chain's bits as ltx_adaln_run does,
    at chains of different widths and timesteps, and refuses bad arguments."""
    import ltx25_b200 as L
    rng = np.random.default_rng(7)
    f = lambda *s, sc=1.0: lib.f32_to_bf16((rng.standard_normal(s) * sc).astype(np.float32))
    chains = []
    for dim, rows in ((96, 9), (64, 2), (96, 1), (40, 4)):
        chains.append(L.AdaLN(f(dim, 256, sc=0.1), f(dim, sc=0.1), f(dim, dim, sc=0.15),
                              f(dim, sc=0.1), f(rows * dim, dim, sc=0.15), None))
    ts = [725.0, 725.0, 312.5, 0.0]
    for threads in (1, 3, 8):
        many = L.adaln_run_many(chains, ts, threads=threads)
        for c, t, (out, emb) in zip(chains, ts, many):
            o1, e1 = c(t, threads=threads)
            assert np.array_equal(out.view(np.uint32), o1.view(np.uint32))
            assert np.array_equal(emb.view(np.uint32), e1.view(np.uint32))
    assert L.adaln_run_many([], []) == []
    lib_ = chains[0].lib
    assert lib_.ltx_adaln_run_many(None, None, None, None, 2, 0) == -1     # LTX_E_NULL
    assert lib_.ltx_adaln_run_many(None, None, None, None, -1, 0) == -2    # LTX_E_SHAPE
    for c in chains:
        c.close()
