"""The multi-GPU final gather without a collective, on one GPU: two processes (the ranks), each
with its own engine; rank 0 exports its 8-bit picture planes through CUDA IPC, rank 1 maps them
and its zjai_synthesize_tiles_q call (its round-robin share of the tiles, from its compacted
latent) stores its cores straight into rank 0's planes. Rank 0 adds its own share; the picture
must equal one process synthesising every tile, bit for bit. The ranks only meet at host
barriers (gloo): no kernel waits on another process."""

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, W, TILE, OVERLAP = 200, 344, 128, 16


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        import synthetic as syn
        import zenjpegai_b200 as zj
        from zenjpegai_b200 import sharding
        from zenjpegai_b200.decoder import Decoder
        torch.cuda.set_device(0)
        eng = zj.Engine(0, arena_bytes=2 << 30)
        py, puv = syn.synthesis_params("sop", 2)
        dec = Decoder(eng, "sop", py, puv)
        lh, lw = -(-H // 16), -(-W // 16)
        ly = syn.laplace_latent(33, "pg/ly", (160, lh, lw), 1.5)
        luv = syn.laplace_latent(33, "pg/luv", (96, lh, lw), 1.5)
        tiles = zj.synthesis_tiles(H, W, lh, lw, TILE, OVERLAP)
        ch, cw = -(-H // 2), -(-W // 2)
        sizes = (H * W, ch * cw, ch * cw)
        buf = torch.full((sum(sizes),), 77, dtype=torch.uint8, device="cuda") if rank == 0 else None
        peer = sharding.PeerPlanes(eng, dist, buf, sizes)
        assert peer.ok
        mine = sharding.shard_tiles(tiles, rank, 2)
        cly, cluv, cmine = sharding.compact_latent(mine, torch.from_numpy(ly).cuda(),
                                                   torch.from_numpy(luv).cuda())
        dec.synthesize_tiles(cly, cluv, cmine, H, W, out=peer.planes, bit_depth=8)
        eng.sync()
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 0:
            got = buf.cpu().numpy()
            ref = dec.synthesize(ly, luv, H, W, tile_size=TILE, overlap=OVERLAP, bit_depth=8)
            want = np.concatenate([p.ravel() for p in ref])
            q.put((bool(np.array_equal(got, want)), int((got != want).sum())))
        dist.barrier()
        peer.close()
        dec.close()
        eng.close()
    finally:
        dist.destroy_process_group()


def test_peer_planes_gather():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    ok, bad = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert ok, "%d samples differ" % bad
