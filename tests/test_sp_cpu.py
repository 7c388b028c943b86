"""The sequence-parallel plan on CPU, over gloo ranks.

tests/sp_np.py restates the CUDA block's sequence (head) parallel split:
video rows sharded for every GEMM and row op, the self-attention and the
video->audio keys exchanged to a head split and back, the audio stream
replicated.  Run as 2 and 4 gloo processes, the rows every rank returns,
stacked in rank order, must equal the unsharded oracle block, and every
rank's audio x must be the same.  tests/test_tp_gpu.py runs the device
path (`sp` mode) on 2 GPUs.
"""
import datetime
import os
import socket

import numpy as np
import pytest

from oracle import block_np, lib

CFG = dict(vdim=512, vheads=4, adim=256, aheads=4, vt=24, at=7, tt=5)
SEED = 43


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    t = block_np.random_block_tensors(CFG["vdim"], CFG["vheads"], CFG["adim"],
                                      CFG["aheads"], seed=SEED)
    ins = block_np.random_block_inputs(CFG, seed=SEED + 1, video_grid=(2, 3, 4))
    return t, ins


def _worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    import sp_np
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        t, ins = _inputs()

        def allgather(arr):
            src = torch.from_numpy(np.ascontiguousarray(arr))
            outs = [torch.empty_like(src) for _ in range(world)]
            dist.all_gather(outs, src)
            return [o.numpy() for o in outs]

        vx, ax = sp_np.block_forward_sp(t, ins["video"], ins["audio"], CFG["vdim"],
                                        CFG["vheads"], CFG["adim"], CFG["aheads"],
                                        rank, world, allgather)
        np.save(os.path.join(out_dir, f"v{rank}.npy"), vx)
        np.save(os.path.join(out_dir, f"a{rank}.npy"), ax)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sequence_parallel_block_equals_the_oracle(tmp_path, world):
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(world, _port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    t, ins = _inputs()
    wv, wa = block_np.block_forward(t, ins["video"], ins["audio"], CFG["vdim"],
                                    CFG["vheads"], CFG["adim"], CFG["aheads"])
    v = np.concatenate([np.load(tmp_path / f"v{r}.npy") for r in range(world)], axis=0)
    a0 = np.load(tmp_path / "a0.npy")
    for r in range(1, world):
        assert np.array_equal(np.load(tmp_path / f"a{r}.npy"), a0)
    assert lib.rel_l2(v, wv) < 1e-5
    assert lib.rel_l2(a0, wa) < 1e-5
    assert lib.rel_l2(v, ins["video"]["x"]) > 1e-2
