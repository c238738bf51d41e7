"""Multi-GPU sharding of a picture's synthesis tiles.

Synthesis tiles are independent (src/decoder/reconstruct.rs:311-313: each reads its own latent
window and writes a disjoint core), so the tiles of one picture shard across ranks with no
data-path collective: tile i runs on rank i mod N (round-robin in raster order, the crate's
tile order). Each rank receives only the latent rows and columns its tiles read
(`compact_latent`). The final gather writes each rank's 8-bit cores straight into rank 0's
picture over NVLink (`PeerPlanes`, CUDA IPC), or, where the planes cannot be shared, every rank
quantises its cores into full-size 8-bit planes that are zero elsewhere and a sum-reduce to
rank 0 reassembles the picture (`gather_cores`; the cores are disjoint, so the sum is exact).
"""

import ctypes

import numpy as np


def shard_tiles(tiles, rank, world):
    """The tiles rank `rank` of `world` synthesises (round-robin over the tile list)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    return [t for i, t in enumerate(tiles) if i % world == rank]


def _merge(ranges):
    """Sorted, merged [a, b) intervals and, per interval, its offset in the compacted axis."""
    out = []
    for a, b in sorted(ranges):
        if out and a <= out[-1][1]:
            out[-1][1] = max(out[-1][1], b)
        else:
            out.append([a, b])
    offs, o = [], 0
    for a, b in out:
        offs.append(o)
        o += b - a
    return out, offs


def compact_latent(tiles, lat_y, lat_uv):
    """The latent rows and columns `tiles` read, packed into smaller latents (numpy arrays or
    torch tensors [c, lh, lw]), and the tiles with their latent windows moved into them; the
    picture coordinates (image, core, offset) are unchanged, so the cores land where they did.
    Returns (lat_y_c, lat_uv_c, tiles_c)."""
    rows, roff = _merge({(t["lat_y"], t["lat_y"] + t["lat_h"]) for t in tiles})
    cols, coff = _merge({(t["lat_x"], t["lat_x"] + t["lat_w"]) for t in tiles})
    ri = np.concatenate([np.arange(a, b) for a, b in rows])
    ci = np.concatenate([np.arange(a, b) for a, b in cols])

    def pick(lat):
        if hasattr(lat, "index_select"):
            import torch
            r = torch.as_tensor(ri, device=lat.device)
            c = torch.as_tensor(ci, device=lat.device)
            return lat.index_select(1, r).index_select(2, c).contiguous()
        return np.ascontiguousarray(lat[:, ri][:, :, ci])

    def move(v, ranges, offs):
        for (a, b), o in zip(ranges, offs):
            if a <= v < b:
                return o + v - a
        raise ValueError("latent window outside the merged ranges")

    out = []
    for t in tiles:
        u = dict(t)
        u["lat_y"] = move(t["lat_y"], rows, roff)
        u["lat_x"] = move(t["lat_x"], cols, coff)
        out.append(u)
    return pick(lat_y), pick(lat_uv), out


class _Ptr:
    """A raw device address where the decoder expects a tensor (it only reads data_ptr())."""

    def __init__(self, p):
        self.p = p

    def data_ptr(self):
        return self.p


class PeerPlanes:
    """Rank 0's 8-bit picture buffer (luma plane, then the two chroma planes, contiguous)
    mapped into every rank through CUDA IPC. `planes` are the plane pointers this rank passes
    as the output of zjai_synthesize_tiles_q: rank 0's own planes on rank 0, the mapped ones
    elsewhere. After each synthesis, `done()` enqueues a one-element all-reduce on the current
    stream, which orders rank 0's later reads after every rank's cores have been written.
    `ok` is False on every rank (and `planes` None) when any rank could not map the planes;
    the caller then gathers with `gather_cores`."""

    def __init__(self, engine, dist, buf, plane_bytes):
        import torch
        from . import _lib
        self.engine, self.dist, self.mapped, self.planes = engine, dist, None, None
        L = _lib.lib()
        msg = [None, None]
        if dist.get_rank() == 0:
            h = (ctypes.c_ubyte * 64)()
            off = ctypes.c_uint64()
            if L.zjai_ipc_export(engine.handle, ctypes.c_void_p(buf.data_ptr()), h,
                                 ctypes.byref(off)) == 0:
                msg = [bytes(h), int(off.value)]
            base = buf.data_ptr()
        dist.broadcast_object_list(msg, src=0)
        ok = msg[0] is not None
        if ok and dist.get_rank() != 0:
            h = (ctypes.c_ubyte * 64).from_buffer_copy(msg[0])
            p = ctypes.c_void_p()
            ok = L.zjai_ipc_import(engine.handle, h, msg[1], ctypes.byref(p)) == 0
            if ok:
                self.mapped = base = p.value
        # every rank agrees on the outcome before any rank relies on it
        dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
        flag = torch.tensor([1 if ok else 0], device=dev, dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        self.ok = bool(flag.item())
        if not self.ok:
            self.close()
            return
        o0, o1, o2 = 0, plane_bytes[0], plane_bytes[0] + plane_bytes[1]
        self.planes = (_Ptr(base + o0), _Ptr(base + o1), _Ptr(base + o2))
        self.flag = torch.zeros(1, device=dev)

    def done(self):
        self.dist.all_reduce(self.flag)

    def close(self):
        from . import _lib
        if self.mapped:
            _lib.lib().zjai_ipc_close(self.engine.handle, ctypes.c_void_p(self.mapped))
            self.mapped = None


def gather_cores(buf, dist, dst=0):
    """Sum-reduce a rank's 8-bit planes (zero outside its cores) onto rank `dst`."""
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        dist.reduce(buf, dst=dst, op=dist.ReduceOp.SUM)
    return buf
