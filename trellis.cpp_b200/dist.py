"""Multi-GPU z-slab sharding of a voxel set with halos of whole z planes over NCCL.

The reference runs on one device and only chunks output rows within it
(src/sparse.cpp:94-118); this module splits the voxels across ranks (one process per GPU).

* :func:`plan_slabs` cuts the z axis into `world` slabs at voxel-count quantiles (whole z
  planes, so every voxel belongs to exactly one rank). Rank r owns z in [z_lo, z_hi) and holds
  `halo` planes of each neighbour: a 3x3x3 submanifold conv at an owned voxel reads only voxels
  within one plane, and two stacked convs read two planes when the first conv's halo rows are
  recomputed locally instead of exchanged.
* The local rows are the owned rows and the halo planes ordered by z, each plane in the input's
  order: [lower halo planes | owned planes | upper halo planes]. A local neighbor map built over
  them gives every owned row exactly its global neighbors (tests check this against the
  single-rank oracle); the halo planes and the edge planes are contiguous ranges (received and
  sent in place), and the interior planes, which need no halo, are one range.
* :func:`exchange_halo` sends the boundary planes to the neighbouring ranks with point-to-point
  send/recv (NCCL over NVLink on GPUs, gloo in the CPU tests) into contiguous buffers and
  scatters them to the halo rows' local positions. Nothing else is communicated: no all-reduce,
  no all-gather.
* :class:`SlabRunner` is the benchmark step on one rank, through the C ABI (tb_dist_*): one NCCL
  exchange of the input's two-plane halo, overlapped with the slab's neighbor map, then
  conv(SiLU) over the owned rows and the nearest halo plane on each side, then conv over the
  owned rows (no exchange between the convs). :func:`plan_slabs` and :func:`exchange_halo` are the host-side
  statement of the same plan and exchange, which the CPU tests run with gloo ranks.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist


@dataclass
class SlabPlan:
    rank: int
    world: int
    z_lo: int                  # owned planes: z_lo <= z < z_hi
    z_hi: int
    owned: np.ndarray          # global row ids of owned voxels, in local order (by z, then input order)
    halo_lo: np.ndarray        # global row ids of the lower halo planes (owned by rank-1), ascending
    halo_hi: np.ndarray        # global row ids of the upper halo planes (owned by rank+1), ascending
    local: np.ndarray          # global row ids of the local rows: owned + halo, ordered by z
    own_local: np.ndarray      # local positions of the owned rows
    send_lo: np.ndarray        # local positions of the lowest owned planes (sent to rank-1), ascending
    send_hi: np.ndarray        # local positions of the highest owned planes (sent to rank+1), ascending
    recv_lo: np.ndarray        # local positions of the lower halo planes (received from rank-1)
    recv_hi: np.ndarray        # local positions of the upper halo planes (received from rank+1)

    @property
    def n_owned(self) -> int:
        return int(self.owned.size)

    @property
    def n_local(self) -> int:
        return int(self.local.size)

    def local_rows(self) -> np.ndarray:
        """Global row id of every local row (by z, then input order)."""
        return self.local


def slab_bounds(z: np.ndarray, world: int) -> np.ndarray:
    """z cut points [world+1] at voxel-count quantiles, on whole planes.

    Every slab gets at least one plane (the voxel sets here span hundreds of planes), so the
    owner of plane z_lo-1 is always rank-1 and of plane z_hi always rank+1."""
    z = np.asarray(z, dtype=np.int64)
    if z.size == 0:
        return np.arange(world + 1, dtype=np.int64)
    zmin, zmax = int(z.min()), int(z.max())
    if zmax - zmin + 1 < world:
        raise ValueError(f"{zmax - zmin + 1} z planes cannot be split into {world} slabs")
    csum = np.cumsum(np.bincount(z - zmin, minlength=zmax - zmin + 1))
    total = int(csum[-1])
    cuts = np.empty(world + 1, dtype=np.int64)
    cuts[0] = zmin
    cuts[world] = zmax + 1
    for r in range(1, world):
        k = int(np.searchsorted(csum, total * r / world, side="left"))   # first plane reaching the quantile
        lo = cuts[r - 1] + 1                                               # at least one plane per slab
        hi = zmax + 1 - (world - r)                                        # leave a plane for each later slab
        cuts[r] = min(max(zmin + k + 1, lo), hi)
    return cuts


def plan_slabs(coords: np.ndarray, world: int, rank: int, halo: int = 1) -> SlabPlan:
    """Slab of `rank` for coords [N,3] (x,y,z) or [N,4] (b,x,y,z); z is the last column. The rank
    holds `halo` planes of each neighbour (planes z_lo-halo .. z_lo-1 and z_hi .. z_hi+halo-1)
    and sends its `halo` edge planes on each side; with halo > 1 every slab must hold at least
    `halo` planes, so that a halo never reaches past the neighbouring slab."""
    z = np.asarray(coords)[:, -1].astype(np.int64)
    cuts = slab_bounds(z, world)
    if halo > 1 and world > 1 and int(np.min(np.diff(cuts))) < halo:
        raise ValueError(f"a slab holds fewer than {halo} planes")
    z_lo, z_hi = int(cuts[rank]), int(cuts[rank + 1])
    owned = np.nonzero((z >= z_lo) & (z < z_hi))[0]
    none = np.zeros(0, np.int64)
    halo_lo = np.nonzero((z >= z_lo - halo) & (z < z_lo))[0] if rank > 0 else none
    halo_hi = np.nonzero((z >= z_hi) & (z < z_hi + halo))[0] if rank < world - 1 else none
    # local order: by plane, and within a plane the input order (a stable sort by z), as
    # tb_dist_partition_zslab orders them: [lower halo planes | plane z_lo .. z_hi-1 | upper halo planes]
    sel = np.sort(np.concatenate([owned, halo_lo, halo_hi]))
    local = sel[np.argsort(z[sel], kind="stable")]
    zl = z[local]
    # a sender packs its boundary planes in local order (by z, then ascending global row), which is
    # the order of the receiver's halo positions for the same planes
    send_lo = np.nonzero((zl >= z_lo) & (zl < z_lo + halo))[0] if rank > 0 else none
    send_hi = np.nonzero((zl >= z_hi - halo) & (zl < z_hi))[0] if rank < world - 1 else none
    recv_lo = np.nonzero(zl < z_lo)[0] if rank > 0 else none
    recv_hi = np.nonzero(zl >= z_hi)[0] if rank < world - 1 else none
    own_local = np.nonzero((zl >= z_lo) & (zl < z_hi))[0]
    owned = local[own_local]
    return SlabPlan(rank, world, z_lo, z_hi, owned, halo_lo, halo_hi, local, own_local, send_lo, send_hi,
                    recv_lo, recv_hi)


def exchange_halo(plan: SlabPlan, x: torch.Tensor, gather, scatter, idx=None, wait: bool = True):
    """Fill the halo rows of the local tensor ``x`` ([n_local, C]) from the neighbouring ranks.

    ``gather(x, idx)`` packs rows ``idx`` of ``x`` into a contiguous tensor and
    ``scatter(x, idx, src)`` writes the rows of ``src`` to rows ``idx`` of ``x`` (index_select /
    index_copy_ on CPU, the library's tb_gather_rows / tb_scatter_rows on GPU). ``idx`` holds
    the plan's send_lo, send_hi, recv_lo, recv_hi positions on ``x``'s device (made here when
    absent). With ``wait=False`` the transfers are only started and a handle is returned; pass it
    to :func:`finish_halo` before reading the halo rows (work enqueued in between overlaps them)."""
    if idx is None:
        idx = [torch.from_numpy(a.astype(np.int32)).to(x.device)
               for a in (plan.send_lo, plan.send_hi, plan.recv_lo, plan.recv_hi)]
    s_lo, s_hi, r_lo, r_hi = idx
    ops = []
    bufs = []
    recvs = []
    # a plane that is empty on one side is empty on the other (it is the same plane), so both
    # ranks skip the same transfers
    if plan.rank > 0 and plan.send_lo.size:
        sb = gather(x, s_lo)
        bufs.append(sb)
        ops.append(dist.P2POp(dist.isend, sb, plan.rank - 1))
    if plan.rank > 0 and plan.recv_lo.size:
        rb = x.new_empty((plan.recv_lo.size,) + tuple(x.shape[1:]))
        recvs.append((r_lo, rb))
        ops.append(dist.P2POp(dist.irecv, rb, plan.rank - 1))
    if plan.rank < plan.world - 1 and plan.send_hi.size:
        sb = gather(x, s_hi)
        bufs.append(sb)
        ops.append(dist.P2POp(dist.isend, sb, plan.rank + 1))
    if plan.rank < plan.world - 1 and plan.recv_hi.size:
        rb = x.new_empty((plan.recv_hi.size,) + tuple(x.shape[1:]))
        recvs.append((r_hi, rb))
        ops.append(dist.P2POp(dist.irecv, rb, plan.rank + 1))
    works = dist.batch_isend_irecv(ops) if ops else []
    handle = (works, bufs, recvs, x, scatter)
    if not wait:
        return handle
    finish_halo(handle)
    return x


def finish_halo(handle) -> None:
    """Wait for the transfers of an ``exchange_halo(..., wait=False)`` call and place the
    received rows."""
    works, _bufs, recvs, x, scatter = handle   # the send buffers stay alive until the sends complete
    for w in works:
        w.wait()
    for pos, rb in recvs:
        scatter(x, pos, rb)


class SlabRunner:
    """The benchmark step on one rank: map + conv(SiLU) + conv on a z-slab, through the C ABI's
    tb_dist_* calls. The slab holds two halo planes per side; one NCCL exchange of the input's
    halo runs while the slab's neighbor map is built, conv 1 computes the owned rows and the
    nearest halo plane on each side (the rows conv 2 reads beyond the slab), and conv 2 the
    owned rows: no exchange between the convs, and each conv is one launch.

    Every rank builds the same global inputs (the generator is seeded alike), so the owned rows
    can be checked against the single-GPU step (:meth:`check_against_single_gpu`)."""

    launches_per_step = 0                 # set in __init__

    halo_planes = 2

    def __init__(self, coords_np: np.ndarray, ci: int, device, generator, uid: bytes):
        from . import ops
        self.ops = ops
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()
        self.device = device
        self.ci = ci
        self.coords_global = torch.from_numpy(np.ascontiguousarray(coords_np)).to(device)
        self.n_total = coords_np.shape[0]
        # the same global features on every rank (same seed); the rank's slab takes its rows
        self.feats_global = torch.randn((self.n_total, ci), device=device, generator=generator).bfloat16()
        self.dist = ops.Dist(device, self.rank, self.world, uid, halo_planes=self.halo_planes)
        self.slab = self.dist.partition(self.coords_global)
        self.rows = self.dist.local_rows().long()
        self.n_local = int(self.slab.n_local)
        self.n_owned = int(self.slab.n_owned)
        self.owned = slice(int(self.slab.owned_begin), int(self.slab.owned_begin) + self.n_owned)
        self.feats = self.feats_global[self.rows].contiguous()
        self.h = torch.zeros((self.n_local, ci), dtype=torch.bfloat16, device=device)
        self.out = torch.zeros((self.n_local, ci), dtype=torch.bfloat16, device=device)
        # our kernels per step: the map and one launch per conv (NCCL's kernel is not counted)
        self.launches_per_step = ops.NBR_MAP_LAUNCHES + 2
        self.graph = None
        self._wl = {}

    def local_weight(self, w):
        """w with its taps in the slab map's order, made once per weight tensor (as a model
        would at load time)."""
        key = (w.data_ptr(), tuple(w.shape), w.dtype)
        if key not in self._wl:
            self._wl[key] = self.dist.local_weight(w)
        return self._wl[key]

    def step(self, w1, w2):
        w1l, w2l = self.local_weight(w1), self.local_weight(w2)
        self.dist.exchange(self.feats)          # overlaps the map build
        self.dist.build_map()
        self.dist.submconv_grow(1, self.feats, w1l, None, epi="silu", out=self.h)
        self.dist.submconv_grow(0, self.h, w2l, None, out=self.out)

    def capture(self, w1, w2, warmup: int = 3) -> None:
        """Record one step (map, both convs and their NCCL halo exchanges) into a CUDA graph.

        With fewer voxels per rank the device work of a step shrinks to a few hundred
        microseconds while issuing it from Python (about twenty launches and two NCCL groups per
        rank, with every rank's process on one host) takes longer; replaying the graph issues the
        whole step at once. Warm-up steps run on a side stream first so that every workspace and
        NCCL connection exists before recording."""
        cur = torch.cuda.current_stream(self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.step(w1, w2)
        cur.wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step(w1, w2)
        torch.cuda.synchronize(self.device)

    def replay(self) -> None:
        """One step from the recorded graph (see :meth:`capture`)."""
        self.graph.replay()

    def count_valid_pairs(self) -> int:
        """Present (voxel, tap) pairs over the owned rows (the algorithmic work of one conv)."""
        return self.dist.count_valid_pairs()

    def check_against_single_gpu(self, w1, w2) -> dict:
        """The whole voxel set's step on this GPU alone (map, conv, conv), compared with the
        owned rows of the sharded step; returns this rank's max|d|/max|ref| and bit-exact rows."""
        ops = self.ops
        n = self.n_total
        nbr = ops.build_neighbor_table(self.coords_global)
        h = ops.sparse_submconv(self.feats_global, nbr, w1, None, epi="silu")
        ref = ops.sparse_submconv(h, nbr, w2, None)
        mine = self.out[self.owned].float()
        want = ref[self.rows[self.owned]].float()
        same = (mine == want).all(dim=1)
        d = (mine - want).abs().max()
        scale = want.abs().max().clamp_min(1e-30)
        ops.check_device()
        res = {"rows_checked": int(self.n_owned), "rows_bit_exact": int(same.sum().item()),
               "max_abs": float(d.item()), "max_ref": float(scale.item())}
        del nbr, h, ref
        assert n == self.coords_global.shape[0]
        return res

    def close(self):
        """Finish the device work and release the recorded graph (it holds NCCL calls and must be
        gone before the communicator), then the dist and its communicator."""
        torch.cuda.synchronize(self.device)
        self.graph = None
        self.dist.close()
