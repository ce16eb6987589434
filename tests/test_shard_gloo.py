"""Batch sharding across ranks (world_size 2, gloo on CPU).

Each rank declares its slice of the global batch and samples parameters for
its own elements only; gathered, they must equal what one process sampling
the whole global batch gets — with no collective in the sampling itself.
The batch-max sigma that sizes Gaussian taps must be the global one."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

GLOBAL_B = 8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sample_all(ba, B):
    torch.manual_seed(0)
    aff = ba.RandAffine(prob=0.7, rotate_range=0.785, shear_range=0.3, translate_range=5,
                        scale_range=0.1).sample_host(B, (B, 1, 16, 16, 16))
    el = ba.Rand3DElastic(prob=1.0, sigma_range=(5.0, 7.0),
                          magnitude_range=(50.0, 150.0)).sample_host(B, (B, 1, 16, 16, 16))
    sm = ba.RandGaussianSmooth(prob=0.5, sigma_x=(0.5, 1.5)).sample_host(B, (B, 1, 16, 16, 16))
    nz = ba.RandGaussianNoise(prob=0.5, std=(0.1, 0.5)).sample_host(B, (B, 1, 16, 16, 16))
    ri = ba.RandRicianNoise(prob=0.5, std=0.3).sample_host(B, (B, 1, 16, 16, 16))
    ss = ba.RandStdShiftIntensity(prob=0.5).sample_host(B, (B, 1, 16, 16, 16))
    sh = ba.RandGaussianSharpen(prob=0.5, sigma1_x=(1.0, 3.0)).sample_host(B, (B, 1, 16, 16, 16))
    lr = ba.RandSimulateLowResolution(prob=0.5).sample_host(B, (B, 1, 16, 16, 16))
    return {"mask": aff["mask"].astype(np.float32), "affine": aff["affine"].reshape(B, -1),
            "el_sigma": el["sigma"], "el_max": np.full(B, el["max_sigma"], np.float32),
            "sm_K": np.full(B, sm["K_sigma_x"], np.float32), "sm_sigma": sm["sigma_x"],
            "nz_std": nz["std"], "nz_seed": np.full(B, nz["noise_seed"] % 2**24, np.float32),
            "ri_std": ri["noise_std"], "ri_mask": ri["mask"].astype(np.float32),
            "ss_factor": ss["factor"], "sh_sigma2": sh["sigma2_x"], "sh_alpha": sh["alpha"],
            "sh_K": np.full(B, sh["K_sigma1_x"], np.float32), "lr_zoom": lr["zoom_factor"]}


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import batchaug_b200 as ba
        local = GLOBAL_B // world
        ba.set_shard(rank * local, GLOBAL_B)
        mine = _sample_all(ba, local)
        gathered = {}
        for k, v in mine.items():
            t = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32))
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)  # test-side gather only
            gathered[k] = torch.cat(parts).numpy()
        if rank == 0:
            np.savez(out_path, **gathered)
    finally:
        dist.destroy_process_group()


def test_two_rank_shard_matches_single_process(tmp_path):
    import batchaug_b200 as ba
    out = str(tmp_path / "gathered.npz")
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, join=True,
                       start_method="spawn")
    got = dict(np.load(out))
    ba.set_shard(0, None)
    ref = _sample_all(ba, GLOBAL_B)
    for k in ref:
        np.testing.assert_array_equal(got[k], np.asarray(ref[k], np.float32), err_msg=k)


def test_shard_context_and_bounds():
    import batchaug_b200 as ba
    assert ba.get_shard() == (0, None)
    with ba.shard(4, 8):
        assert ba.get_shard() == (4, 8)
        with pytest.raises(ValueError):
            ba.Rand3DElastic(prob=1.0).sample_host(8, (8, 1, 4, 4, 4))  # 4+8 > 8
    assert ba.get_shard() == (0, None)
    with pytest.raises(ValueError):
        ba.set_shard(-1)
