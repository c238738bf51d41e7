"""Multi-GPU sharding of a picture's synthesis tiles.

Synthesis tiles are independent (src/decoder/reconstruct.rs:311-313: each reads its own latent
window and writes a disjoint core), so the tiles of one picture shard across ranks with no
data-path collective: tile i runs on rank i mod N (round-robin in raster order, the crate's
tile order). The only exchange is the final gather: every rank quantises its cores into
full-size 8-bit planes that are zero elsewhere, and a sum-reduce to rank 0 reassembles the
picture (the cores are disjoint, so the sum is exact).
"""


def shard_tiles(tiles, rank, world):
    """The tiles rank `rank` of `world` synthesises (round-robin over the tile list)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    return [t for i, t in enumerate(tiles) if i % world == rank]


def gather_cores(buf, dist, dst=0):
    """Sum-reduce a rank's 8-bit planes (zero outside its cores) onto rank `dst`."""
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        dist.reduce(buf, dst=dst, op=dist.ReduceOp.SUM)
    return buf
