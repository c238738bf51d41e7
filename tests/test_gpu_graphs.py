"""CUDA graphs of repeated tiled-synthesis calls (zjai_ctx_set_graphs): replays equal the eager
calls bit for bit (several tile shape groups, so the captured call forks and joins the group
streams), see new latent contents at the same pointers, count their kernel launches, and are
dropped when a network is destroyed."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_graph_replay_equals_eager():
    import torch
    import synthetic as syn
    import zenjpegai_b200 as zj
    from zenjpegai_b200.decoder import Decoder
    eng = zj.Engine(0, arena_bytes=8 << 30)
    try:
        py, puv = syn.synthesis_params("hop", 4)
        dec = Decoder(eng, "hop", py, puv)
        H, W = 336, 600  # tiles of 256 / 16: interior, right, bottom and corner shapes
        lh, lw = -(-H // 16), -(-W // 16)
        ly = torch.from_numpy(syn.laplace_latent(5, "ly", (160, lh, lw), 1.5)).cuda()
        luv = torch.from_numpy(syn.laplace_latent(5, "luv", (96, lh, lw), 1.5)).cuda()
        tiles = zj.synthesis_tiles(H, W, lh, lw, 256, 16)
        assert len({(t["img_w"], t["img_h"]) for t in tiles}) == 4
        out = tuple(torch.zeros(s, dtype=torch.uint8, device="cuda")
                    for s in ((H, W), (-(-H // 2), -(-W // 2)), (-(-H // 2), -(-W // 2))))

        def run():
            for o in out:
                o.zero_()
            dec.synthesize_tiles(ly, luv, tiles, H, W, out=out, bit_depth=8)
            eng.sync()
            return [o.cpu().numpy().copy() for o in out]

        eager = run()
        eng.set_graphs(True)
        n0 = eng.launch_count
        first = run()            # eager, records the shape groups
        n1 = eng.launch_count
        captured = run()         # captured and launched
        n2 = eng.launch_count
        replay = run()           # replayed
        n3 = eng.launch_count
        for a, b, c in zip(eager, captured, replay):
            assert np.array_equal(a, b) and np.array_equal(a, c)
        assert n2 - n1 == n3 - n2 > 0 and n1 - n0 > 0
        # new contents at the same pointers: the replay computes them
        ly.mul_(0.5)
        luv.mul_(0.5)
        replay2 = run()
        eng.set_graphs(False)
        eager2 = run()
        for a, b in zip(replay2, eager2):
            assert np.array_equal(a, b)
        assert any(not np.array_equal(a, b) for a, b in zip(replay2, replay))
        # destroying a network drops the graphs (a new network is never served a stale one)
        eng.set_graphs(True)
        run()
        run()
        dec.close()
        dec2 = Decoder(eng, "hop", *syn.synthesis_params("hop", 9))
        dec = dec2
        got = [None]
        for _ in range(3):
            for o in out:
                o.zero_()
            dec.synthesize_tiles(ly, luv, tiles, H, W, out=out, bit_depth=8)
            eng.sync()
            got = [o.cpu().numpy().copy() for o in out]
        eng.set_graphs(False)
        for o in out:
            o.zero_()
        dec.synthesize_tiles(ly, luv, tiles, H, W, out=out, bit_depth=8)
        eng.sync()
        for a, o in zip(got, out):
            assert np.array_equal(a, o.cpu().numpy())
        dec.close()
    finally:
        eng.close()
