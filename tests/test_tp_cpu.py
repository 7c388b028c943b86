"""The tensor-parallel plan on CPU, over gloo ranks.

tests/tp_np.py restates the CUDA block's Megatron sharding (heads split for
q/k/v and the gates, K split for the output projections and ff.net.2, the
q/k RMSNorm's sums of squares and the partial products reduced over ranks).
Run as 2 and 4 gloo processes, every rank must end with the same x, equal to
the unsharded oracle block up to summation order.  This is the host-side
logic the GPU tensor-parallel path follows; tests/test_tp_gpu.py runs the
device path itself on 2 GPUs.
"""
import datetime
import os
import socket

import numpy as np
import pytest

from oracle import block_np, lib, lora_np

CFG = dict(vdim=512, vheads=4, adim=256, aheads=4, vt=24, at=7, tt=5)
SEED = 41
# Adapted sites: column-split (q, k, v, gate logits, ff in), row-split
# (to_out.0, ff.net.2), both streams and the cross attentions.
LORA_MODULES = ["attn1.to_q", "attn1.to_v", "attn1.to_out.0", "attn1.to_gate_logits",
                "attn2.to_k", "ff.net.0.proj", "ff.net.2", "audio_attn1.to_k",
                "audio_ff.net.2", "audio_to_video_attn.to_out.0", "video_to_audio_attn.to_q"]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    t = block_np.random_block_tensors(CFG["vdim"], CFG["vheads"], CFG["adim"],
                                      CFG["aheads"], seed=SEED)
    ins = block_np.random_block_inputs(CFG, seed=SEED + 1, video_grid=(2, 3, 4))
    return t, ins


def _lora(t):
    """module -> (A, B) f32 values, deterministic, shaped like the base."""
    out = {}
    for i, m in enumerate(LORA_MODULES):
        n, k = np.shape(t[m + ".weight"])
        a, b = lora_np.make_pair(np.random.default_rng(SEED * 100 + i), 3 + i, k, n)
        out[m] = (lib.bf16_to_f32(a), lib.bf16_to_f32(b))
    return out


def _folded(t, pairs):
    """The block's tensors with every pair folded into its weight."""
    f = dict(t)
    for m, (a, b) in pairs.items():
        f[m + ".weight"] = lora_np.fold(t[m + ".weight"], a, b)
    return f


def _worker(rank, world, port, out_dir, adapted=False, rows=False):
    import torch
    import torch.distributed as dist
    import tp_np
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        t, ins = _inputs()

        def allreduce(arr):
            dist.all_reduce(torch.from_numpy(arr))

        def allgather(local):
            parts = [torch.empty(local.shape, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(local, np.float32)))
            return np.concatenate([p.numpy() for p in parts], axis=0)

        if rows:
            vx, ax = tp_np.block_forward_tp_rows(t, ins["video"], ins["audio"], CFG["vdim"],
                                                 CFG["vheads"], CFG["adim"], CFG["aheads"],
                                                 rank, world, allreduce, allgather)
        else:
            vx, ax = tp_np.block_forward_tp(t, ins["video"], ins["audio"], CFG["vdim"],
                                            CFG["vheads"], CFG["adim"], CFG["aheads"],
                                            rank, world, allreduce,
                                            lora=_lora(t) if adapted else None)
        np.save(os.path.join(out_dir, f"v{rank}.npy"), vx)
        np.save(os.path.join(out_dir, f"a{rank}.npy"), ax)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,adapted", [(2, False), (4, False), (2, True), (4, True)])
def test_sharded_block_equals_the_oracle(tmp_path, world, adapted):
    """Adapted: each rank applies its share of the full adapters; the oracle
    runs the unsharded block with W += B A (the reference's fold)."""
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(world, _port(), str(tmp_path), adapted), nprocs=world,
                       join=True, start_method="spawn")
    t, ins = _inputs()
    tw = _folded(t, _lora(t)) if adapted else t
    wv, wa = block_np.block_forward(tw, ins["video"], ins["audio"], CFG["vdim"],
                                    CFG["vheads"], CFG["adim"], CFG["aheads"])
    v0 = np.load(tmp_path / "v0.npy")
    a0 = np.load(tmp_path / "a0.npy")
    for r in range(1, world):
        assert np.array_equal(np.load(tmp_path / f"v{r}.npy"), v0)
        assert np.array_equal(np.load(tmp_path / f"a{r}.npy"), a0)
    assert lib.rel_l2(v0, wv) < 1e-5
    assert lib.rel_l2(a0, wa) < 1e-5
    # and the sharding is not vacuous: the block moved x
    assert lib.rel_l2(v0, ins["video"]["x"]) > 1e-2
    if adapted:   # nor are the adapters: the unadapted block differs
        pv, pa = block_np.block_forward(t, ins["video"], ins["audio"], CFG["vdim"],
                                        CFG["vheads"], CFG["adim"], CFG["aheads"])
        assert lib.rel_l2(v0, pv) > 1e-3 and lib.rel_l2(a0, pa) > 1e-3


@pytest.mark.parametrize("world", [2, 4])
def test_row_sharded_residual_equals_the_oracle(tmp_path, world):
    """Tensor parallel with the video residual kept by token rows (reduce-
    scatter / all-gather; the GPU path's default when the tokens split
    evenly): every rank ends with the same whole x, equal to the unsharded
    oracle block up to summation order."""
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(world, _port(), str(tmp_path), False, True),
                       nprocs=world, join=True, start_method="spawn")
    t, ins = _inputs()
    wv, wa = block_np.block_forward(t, ins["video"], ins["audio"], CFG["vdim"],
                                    CFG["vheads"], CFG["adim"], CFG["aheads"])
    v0 = np.load(tmp_path / "v0.npy")
    a0 = np.load(tmp_path / "a0.npy")
    for r in range(1, world):
        assert np.array_equal(np.load(tmp_path / f"v{r}.npy"), v0)
        assert np.array_equal(np.load(tmp_path / f"a{r}.npy"), a0)
    assert lib.rel_l2(v0, wv) < 1e-5
    assert lib.rel_l2(a0, wa) < 1e-5
    assert lib.rel_l2(v0, ins["video"]["x"]) > 1e-2


@pytest.mark.parametrize("adapted", [False, True])
def test_one_rank_plan_is_the_oracle(adapted):
    import tp_np
    t, ins = _inputs()
    pairs = _lora(t) if adapted else None
    vx, ax = tp_np.block_forward_tp(t, ins["video"], ins["audio"], CFG["vdim"],
                                    CFG["vheads"], CFG["adim"], CFG["aheads"], 0, 1,
                                    lambda a: None, lora=pairs)
    tw = _folded(t, pairs) if adapted else t
    wv, wa = block_np.block_forward(tw, ins["video"], ins["audio"], CFG["vdim"],
                                    CFG["vheads"], CFG["adim"], CFG["aheads"])
    assert lib.rel_l2(vx, wv) < 1e-6 and lib.rel_l2(ax, wa) < 1e-6
