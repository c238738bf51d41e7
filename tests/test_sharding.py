"""The multi-GPU sharding logic on CPU: two gloo ranks each synthesise their round-robin share
of a tiled picture (with the CPU oracle standing in for the GPU), quantise their cores into
zero-elsewhere 8-bit planes, and the sum-reduce onto rank 0 reproduces the single-process
picture bit for bit. Also: the shard partition covers every tile exactly once for N = 1..8.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as zo
from zenjpegai_b200 import sharding
import synthetic as syn

H, W, TILE, OVERLAP = 160, 272, 96, 16


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _picture():
    lh, lw = -(-H // 16), -(-W // 16)
    ly = syn.laplace_latent(31, "shard/ly", (160, lh, lw), 1.5)
    luv = syn.laplace_latent(31, "shard/luv", (96, lh, lw), 1.5)
    py, puv = syn.synthesis_params("sop", 2)
    return ly, luv, py, puv


def _synth_tiles(tiles, ly, luv, py, puv):
    """reconstruct.rs:379-464 for a subset of tiles, via the oracle, into zeroed planes."""
    cky, ckuv = zo.Checkpoint(py), zo.Checkpoint(puv)
    ry = np.zeros((H, W), np.float32)
    ch, cw = -(-H // 2), -(-W // 2)
    ru = np.zeros((ch, cw), np.float32)
    rv = np.zeros((ch, cw), np.float32)
    for t in tiles:
        wl = ly[:, t["lat_y"]:t["lat_y"] + t["lat_h"], t["lat_x"]:t["lat_x"] + t["lat_w"]]
        wc = luv[:, t["lat_y"]:t["lat_y"] + t["lat_h"], t["lat_x"]:t["lat_x"] + t["lat_w"]]
        oy = zo.synthesis_primary(cky, zo.SOP, wl, t["img_h"], t["img_w"])[0]
        ouv = zo.synthesis_secondary(ckuv, zo.SOP, wl, wc, t["img_h"], t["img_w"])
        cy, cx, hh, ww = t["core_y"], t["core_x"], t["core_h"], t["core_w"]
        ry[cy:cy + hh, cx:cx + ww] = oy[t["off_y"]:t["off_y"] + hh, t["off_x"]:t["off_x"] + ww]
        for c, dst in enumerate((ru, rv)):
            for py_ in range(-(-cy // 2) * 2, cy + hh, 2):
                for px_ in range(-(-cx // 2) * 2, cx + ww, 2):
                    dst[py_ // 2, px_ // 2] = ouv[c, t["off_y"] + py_ - cy,
                                                 t["off_x"] + px_ - cx]
    return ry, ru, rv


def _pack8(ry, ru, rv):
    return torch.from_numpy(np.concatenate([zo.quantize_plane(p).astype(np.uint8).ravel()
                                            for p in (ry, ru, rv)]))


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ly, luv, py, puv = _picture()
        tiles = zo.synthesis_tiles(H, W, ly.shape[1], ly.shape[2], TILE, OVERLAP)
        mine = sharding.shard_tiles(tiles, rank, world)
        # the rank receives only the latent rows / columns its tiles read
        cly, cluv, cmine = sharding.compact_latent(mine, ly, luv)
        buf = _pack8(*_synth_tiles(cmine, cly, cluv, py, puv))
        sharding.gather_cores(buf, dist)
        if rank == 0:
            q.put(buf.numpy().copy())
    finally:
        dist.destroy_process_group()


def test_shard_partition():
    tiles = zo.synthesis_tiles(2160, 3840, 135, 240, 512, 16)
    for world in range(1, 9):
        seen = []
        for r in range(world):
            seen += [id(t) for t in sharding.shard_tiles(tiles, r, world)]
        assert sorted(seen) == sorted(id(t) for t in tiles)
    with pytest.raises(ValueError):
        sharding.shard_tiles(tiles, 2, 2)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_compact_latent_windows(world):
    """Every tile's latent window read from its rank's compacted latent equals the window of
    the full latent (4K config-4 tiling), and the compacted latent is no larger than needed."""
    lh, lw = 135, 240
    ly = syn.laplace_latent(32, "cl/ly", (160, lh, lw), 1.5)
    luv = syn.laplace_latent(32, "cl/luv", (96, lh, lw), 1.5)
    tiles = zo.synthesis_tiles(2160, 3840, lh, lw, 512, 16)
    for r in range(world):
        mine = sharding.shard_tiles(tiles, r, world)
        cly, cluv, cmine = sharding.compact_latent(mine, ly, luv)
        for t, u in zip(mine, cmine):
            for k in ("img_x", "img_y", "core_x", "core_y", "core_w", "core_h", "lat_w", "lat_h"):
                assert t[k] == u[k]
            for full, comp in ((ly, cly), (luv, cluv)):
                a = full[:, t["lat_y"]:t["lat_y"] + t["lat_h"], t["lat_x"]:t["lat_x"] + t["lat_w"]]
                b = comp[:, u["lat_y"]:u["lat_y"] + u["lat_h"], u["lat_x"]:u["lat_x"] + u["lat_w"]]
                assert np.array_equal(a, b)
        cols = len({x for t in mine for x in range(t["lat_x"], t["lat_x"] + t["lat_w"])})
        rows = len({y for t in mine for y in range(t["lat_y"], t["lat_y"] + t["lat_h"])})
        assert cly.shape == (160, rows, cols)
        if world == 8:
            assert cly.shape[2] <= 32  # one tile column: 1/7.5 of the latent


def test_two_rank_gather_reproduces_picture():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ly, luv, py, puv = _picture()
    want = zo.synthesize(zo.Checkpoint(py), zo.Checkpoint(puv), zo.SOP, ly, luv, H, W,
                         tile_size=TILE, overlap=OVERLAP)
    assert np.array_equal(got, _pack8(*want).numpy())
