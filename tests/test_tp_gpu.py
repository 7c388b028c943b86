"""Multi-GPU block and stack on 2 GPUs (BASELINE config 5's multi-GPU leg),
tensor parallel (ltx_ctx_set_tp) and sequence parallel (ltx_ctx_set_sp),
against the one-GPU block and the CPU oracle.

Two spawned processes, one per GPU, join one NCCL group (rendezvous id made
here), load the same full weights (tensor parallel: each keeps its shard;
sequence parallel: each keeps them whole and runs half the video tokens),
and run a block and a 2-block stack on the same replicated inputs.  Tensor
parallel runs with the residual sharded by token rows (the default when the
tokens split evenly) and, in tp_allreduce, with x whole on every rank and the
products all-reduced, in tp_chunked with the feed-forward as two token
chunks whose collectives overlap the other chunk's GEMMs (the default from 8
ranks), and in tp_scatter with the row-split products reduce-scattered by
the GEMM itself (each row's partial stored into its owner's receive slot over
peer memory, then summed by the owner).  Checked: both ranks end with the same x; it matches the
oracle at the block bars of tests/test_block_gpu.py and the one-GPU device
block within bf16.  Skipped with fewer than 2 GPUs.  NVLS is off in the
workers, and a worker that does not finish in time is killed by PID.
"""
import os

import numpy as np
import pytest

from oracle import block_np, lib, lora_np

from test_block_gpu import DELTA_BAR, OUT_BAR, bf16r, host, to_dev

pytestmark = pytest.mark.gpu

CFG = dict(vdim=512, vheads=4, adim=256, aheads=4, vt=24, at=7, tt=5)
SEED = 61
WORLD = 2


def _setup():
    t = block_np.random_block_tensors(CFG["vdim"], CFG["vheads"], CFG["adim"],
                                      CFG["aheads"], seed=SEED)
    t2 = block_np.random_block_tensors(CFG["vdim"], CFG["vheads"], CFG["adim"],
                                       CFG["aheads"], seed=SEED + 7)
    ins = block_np.random_block_inputs(CFG, seed=SEED + 1, video_grid=(2, 3, 4))
    for s in ("video", "audio"):
        for key in ("x", "context", "timesteps", "cross_scale_shift", "cross_gate",
                    "prompt_timestep"):
            ins[s][key] = bf16r(ins[s][key])
    return t, t2, ins


# Adapted modules for the *_lora modes: column-split sites (q, gate, ff in,
# the fused k/v), row-split ones (to_out.0, ff.net.2) and the cross
# attentions' audio-width sites.
LORA_MODULES = ["attn1.to_q", "attn1.to_out.0", "attn1.to_gate_logits", "attn2.to_v",
                "ff.net.0.proj", "ff.net.2", "audio_attn1.to_k", "audio_ff.net.2",
                "audio_to_video_attn.to_out.0", "video_to_audio_attn.to_v"]


def _pairs(t, seed):
    """module -> (a bits, b bits), deterministic, shaped like the base."""
    out = {}
    for i, m in enumerate(LORA_MODULES):
        n, k = np.shape(t[m + ".weight"])
        out[m] = lora_np.make_pair(np.random.default_rng(seed * 100 + i), 5 + i, k, n)
    return out


def _run(ctx, world_blocks, ins, lora=False):
    """One block forward, then a stack of all blocks from the same inputs."""
    import torch
    import ltx25_b200 as L
    blocks = []
    deqs = []
    for bi, t in enumerate(world_blocks):
        b = L.Block(ctx, CFG["vdim"], CFG["vheads"], CFG["adim"], CFG["aheads"])
        deqs.append(b.load(t))
        if lora:
            for m, (a, bb) in _pairs(t, bi).items():
                dev = lambda x: torch.from_numpy(np.asarray(x, np.uint16).view(np.int16)).cuda() \
                    .view(torch.bfloat16)
                b.set_lora(m, L.Lora(ctx, dev(a), dev(bb)))
        b.finalize()
        blocks.append(b)
    blocks[0].reserve(CFG["vt"], CFG["at"], CFG["tt"])
    dv, da = to_dev(ins["video"]), to_dev(ins["audio"])
    blocks[0].forward(dv, da)
    torch.cuda.synchronize()
    ctx.check()
    one = (host(dv["x"]), host(da["x"]))
    st = L.Stack(ctx, blocks)
    st.reserve(CFG["vt"], CFG["at"], CFG["tt"])
    dv, da = to_dev(ins["video"]), to_dev(ins["audio"])
    st.forward(dv, da)
    torch.cuda.synchronize()
    ctx.check()
    two = (host(dv["x"]), host(da["x"]))
    st.close()
    for b in blocks:
        b.close()
    return one, two, deqs


def _worker(rank, world, uid, out_dir, mode):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    if mode.startswith("tp_allreduce"):
        # the whole-x layout (all-reduced products) instead of the default
        # row-sharded residual (reduce-scatter / all-gather)
        os.environ["LTX25_TP_ROWS"] = "0"
    if mode.startswith("tp_chunked"):
        # the row-sharded feed-forward as two token chunks whose collectives
        # overlap the other chunk's GEMMs (the default from 8 ranks)
        os.environ["LTX25_TP_FF_CHUNKS"] = "1"
    # the fused reduce-scatter (the row-split GEMMs store each row's partial
    # into its owner's receive slot over peer memory) is the default; the
    # other row-sharded modes run the NCCL reduce-scatter
    os.environ["LTX25_TP_SCATTER"] = "1" if mode.startswith("tp_scatter") else "0"
    import torch
    import ltx25_b200 as L
    torch.cuda.set_device(rank)
    ctx = L.Context(rank)
    (ctx.set_tp if mode.startswith("tp") else ctx.set_sp)(rank, world, uid)
    t, t2, ins = _setup()
    one, two, _ = _run(ctx, [t, t2], ins, lora=mode.endswith("lora"))
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), v1=one[0], a1=one[1], v2=two[0], a2=two[1])
    ctx.close()


@pytest.mark.parametrize("mode", ["tp", "sp", "tp_lora", "sp_lora", "tp_allreduce",
                                  "tp_chunked", "tp_chunked_lora", "tp_scatter",
                                  "tp_scatter_lora"])
def test_two_gpu_block_and_stack(ctx, tmp_path, mode):
    import torch
    import torch.multiprocessing as mp
    import ltx25_b200 as L
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    uid = L.tp_unique_id()
    pc = mp.start_processes(_worker, args=(WORLD, uid, str(tmp_path), mode), nprocs=WORLD,
                            join=False, start_method="spawn")
    try:
        for _ in range(60):
            if pc.join(timeout=10):
                break
        else:
            raise AssertionError("tensor-parallel workers did not finish in 600 s")
    finally:
        for p in pc.processes:
            if p.is_alive():
                p.kill()
    r = [np.load(tmp_path / f"r{k}.npz") for k in range(WORLD)]
    for k in range(1, WORLD):
        for key in ("v1", "a1", "v2", "a2"):
            assert np.array_equal(r[k][key], r[0][key]), f"rank {k} {key} differs"

    # one GPU, same weights, adapters and inputs
    lora = mode.endswith("lora")
    t, t2, ins = _setup()
    one, two, deqs = _run(ctx, [t, t2], ins, lora=lora)

    def eff(t, deq):
        import ltx25_b200 as L
        ow = {}
        for k, v in deq.items():
            if L.is_quantized_name(k, np.ndim(t[k])):
                ow[k] = v
            elif k.endswith(".bias") or "to_gate_logits" in k:
                ow[k] = bf16r(v)
            else:
                ow[k] = v
        return ow

    ow = eff(t, deqs[0])
    if lora:   # the oracle runs the folded weights (W += B A)
        for m, (a, bb) in _pairs(t, 0).items():
            ow[m + ".weight"] = lora_np.fold(ow[m + ".weight"], lib.bf16_to_f32(a),
                                             lib.bf16_to_f32(bb))
    wv, wa = block_np.block_forward(ow, ins["video"], ins["audio"], CFG["vdim"], CFG["vheads"],
                                    CFG["adim"], CFG["aheads"])
    bv, ba = block_np.block_forward(ow, ins["video"], ins["audio"], CFG["vdim"], CFG["vheads"],
                                    CFG["adim"], CFG["aheads"], x_round=bf16r)
    for name, got, g1, want, wantb, x0 in (
            ("video", r[0]["v1"], one[0], wv, bv, ins["video"]["x"]),
            ("audio", r[0]["a1"], one[1], wa, ba, ins["audio"]["x"])):
        out_r = lib.rel_l2(got, want)
        delta_r = lib.rel_l2(got - x0, wantb - x0)
        vs1 = lib.rel_l2(got - x0, g1 - x0)
        print(name, out_r, delta_r, vs1)
        # adapted: the reference's adapter bar (tests/ltx25-lora-apply-test.cc:681)
        ob, db = (4e-2, 4e-2) if lora else (OUT_BAR, DELTA_BAR)
        assert out_r < ob and delta_r < db, (name, out_r, delta_r)
        assert vs1 < DELTA_BAR, (name, vs1)
    for name, got, g1 in (("video", r[0]["v2"], two[0]), ("audio", r[0]["a2"], two[1])):
        vs1 = lib.rel_l2(got, g1)
        print("stack", name, vs1)
        assert vs1 < (DELTA_BAR if lora else OUT_BAR), (name, vs1)
