"""Spatial domain decomposition of one periodic system over ranks (one GPU per rank).

The reference's multi-GPU inference (``cli/inference_ddp.py:143-340``) partitions atoms by
region and exchanges ghost-atom features after every layer.  Both exchange patterns are here:
:func:`layer_exchange_step` does that (a one-cutoff halo, the ictd engine run in steps, ghost
feature rows exchanged after every layer and their gradients returned in the reverse pass);
:func:`decomposed_step` recomputes the ghosts redundantly over a receptive-field halo, with no
per-layer communication.  The notes below describe the latter; both share the halo exchange.

* The cell is cut into a ``(px, py, pz)`` grid of blocks; rank ``r`` owns the atoms of one block
  (in practice: whatever atoms the caller hands it; only their bounding box matters).
* Once per step every rank receives every periodic image of any rank's atoms (its own included)
  that lies within the halo width ``h`` of its owned atoms' bounding box along the split axes.
  With ``h >= num_interaction * cutoff`` the energy of every owned atom is exact: its receptive
  field is ``num_interaction`` hops of ``cutoff``.
* The local system is [owned atoms | ghost images], open along split axes (the ghosts are
  explicit images) and periodic along the others.  The engine evaluates
  ``E_local = sum of owned atom energies`` (``num_local`` convention) and ``-dE_local/dpos`` for
  all local atoms.
* Ghost forces go back to their owners and are added (the one reverse exchange); energies and
  virials are summed over ranks (``W = sum_r sum_{e in rank r} r_e (x) dE_r/dr_e``).

A step is written once, as a generator that yields its collectives as requests
(``("all_gather", t)``, ``("all_reduce_sum", t)``, ``("all_to_all", (rows, counts, recv_counts))``);
:func:`run_dist` serves them with ``torch.distributed`` (NCCL on GPUs, gloo on CPU; variable
lengths through ``all_to_all_single``) and :func:`run_local` serves all ranks of a decomposition
in one process, which is how one device tests the whole multi-rank path.  The steps also yield
``("mark", "begin" | "end")`` around their halo phases (the halo plan with its position exchange,
the per-layer feature and gradient exchanges, the reverse force exchange): with ``HALO_TIMER``
set to a list, :func:`run_dist` records a CUDA event at each mark into it (``halo_ms`` of
``bench.py``); otherwise marks cost nothing.
"""

from __future__ import annotations

import itertools
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

import numpy as np
import torch


def grid_for(world: int) -> tuple:
    """Default block grid for a world size: 1 -> 1x1x1, 2 -> 2x1x1, 4 -> 2x2x1, 8 -> 2x2x2 ..."""
    dims = [1, 1, 1]
    k = 0
    w = world
    while w > 1:
        if w % 2:
            raise ValueError(f"world size {world} is not a power of two; pass dims explicitly")
        dims[k % 3] *= 2
        w //= 2
        k += 1
    return tuple(dims)


def block_of(rank: int, dims: Sequence[int]) -> tuple:
    """Block coordinates of a rank (row-major over the (px, py, pz) grid)."""
    px, py, pz = dims
    return (rank // (py * pz), (rank // pz) % py, rank % pz)


@dataclass
class Decomposition:
    """Static description of the decomposition (identical on every rank)."""

    cell: np.ndarray                # (3, 3) row-vector lattice of the periodic system
    dims: Sequence[int]             # blocks per axis
    halo: float                     # ghost halo width in Angstrom (>= num_interaction * cutoff)
    split: tuple = field(init=False)

    def __post_init__(self):
        self.cell = np.asarray(self.cell, dtype=np.float64).reshape(3, 3)
        self.dims = tuple(int(d) for d in self.dims)
        self.split = tuple(d > 1 for d in self.dims)
        for k in range(3):
            if not self.split[k]:
                continue
            if any(self.cell[k, j] != 0.0 for j in range(3) if j != k) or any(
                    self.cell[j, k] != 0.0 for j in range(3) if j != k):
                raise ValueError("a split axis needs an axis-aligned cell vector orthogonal to the others")
            if not (2.0 * self.halo < self.cell[k, k]):
                raise ValueError("the halo must be shorter than half the cell along a split axis "
                                 "(only the nearest periodic images are exchanged)")

    @property
    def world(self) -> int:
        return int(np.prod(self.dims))

    @property
    def local_pbc(self) -> tuple:
        """Periodicity of a rank's local system: open along split axes."""
        return tuple(not s for s in self.split)

    def block_of(self, rank: int) -> tuple:
        return block_of(rank, self.dims)

    def block_bounds(self, rank: int) -> np.ndarray:
        """(2, 3) Cartesian bounds of a rank's block (axis-aligned split axes; others: full cell)."""
        b = self.block_of(rank)
        lo, hi = np.zeros(3), np.zeros(3)
        for k in range(3):
            L = self.cell[k, k] if self.cell[k, k] > 0 else 0.0
            lo[k] = L * b[k] / self.dims[k]
            hi[k] = L * (b[k] + 1) / self.dims[k]
        return np.stack([lo, hi])

    def images(self) -> List[tuple]:
        """Image shifts S (in cell vectors) that can place an atom in another rank's halo."""
        rng = [(-1, 0, 1) if s else (0,) for s in self.split]
        return list(itertools.product(*rng))


# ---------------------------------------------------------------------------- collectives
def all_gather(t: torch.Tensor):
    """(world, *t.shape) stack of every rank's ``t``."""
    return (yield ("all_gather", t))


def all_reduce_sum(t: torch.Tensor):
    return (yield ("all_reduce_sum", t))


def all_to_all(rows: torch.Tensor, counts: List[int], recv_counts: Optional[List[int]] = None):
    """Rows ``rows[sum(counts[:d]) : sum(counts[:d + 1])]`` go to rank d; returns
    ``(received rows grouped by source rank, recv_counts)``."""
    return (yield ("all_to_all", (rows, list(counts), recv_counts)))


HALO_TIMER: Optional[list] = None  # (mark, torch.cuda.Event) pairs recorded by run_dist when a list


def halo_mark(which: str):
    yield ("mark", which)


class RankFailure(RuntimeError):
    """Another rank of the decomposition failed, or never arrived at a step: raised by
    :meth:`StepGuard.begin` before this rank enters the step's first collective."""


class StepGuard:
    """Failure detection between steps through a key-value store shared by the ranks (a
    ``torch.distributed`` store, e.g. the ``TCPStore`` of the job), independent of the process
    group whose collectives it protects.

    :meth:`begin` starts a step: the rank adds itself to the step's arrival count and waits until
    all ``world`` ranks have arrived, a rank has posted a failure, or ``timeout`` seconds pass.  A
    rank whose step raises posts the reason (:meth:`fail`; :func:`run_dist` does it), so the other
    ranks learn of it on the host before their next step's first collective instead of waiting in
    that collective until the process group's own timeout; a rank that stops without posting shows
    up as a missing arrival.  A rank that fails between two collectives of a step leaves its peers
    in the collective in flight: the process group's timeout (set it short) ends that one with an
    error, and the posted reason tells the peers which rank failed and why.  The first failure
    posted is the one kept.  Rank 0 deletes a step's arrival key once every rank has passed the
    next step's arrival."""

    def __init__(self, store, rank: int, world: int, timeout: float = 60.0, prefix: str = "fsctep_step_guard",
                 poll: float = 1e-3):
        self.store, self.rank, self.world = store, int(rank), int(world)
        self.timeout, self.prefix, self.poll = float(timeout), prefix, float(poll)
        self.step = 0

    def _fail_key(self) -> str:
        return f"{self.prefix}/failed"

    def failure(self) -> Optional[str]:
        """The failure posted by any rank, or None."""
        key = self._fail_key()
        if not self.store.check([key]):
            return None
        msg = self.store.get(key)
        msg = msg.decode() if isinstance(msg, (bytes, bytearray)) else str(msg)
        return msg or None

    def fail(self, reason: str) -> None:
        """Post this rank's failure (kept only if no rank posted one before)."""
        self.store.compare_set(self._fail_key(), "", f"rank {self.rank}: {reason}")

    def begin(self) -> None:
        """Arrival at the next step; raises RankFailure if a rank failed or did not arrive."""
        msg = self.failure()
        if msg:
            raise RankFailure(msg)
        self.step += 1
        key = f"{self.prefix}/arrived/{self.step}"
        self.store.add(key, 1)
        t0 = time.monotonic()
        while True:
            n = self.store.add(key, 0)
            if n >= self.world:
                break
            msg = self.failure()
            if msg:
                raise RankFailure(msg)
            if time.monotonic() - t0 > self.timeout:
                msg = (f"step {self.step}: {self.world - n} of {self.world} ranks did not arrive within "
                       f"{self.timeout:g} s")
                self.fail(msg)
                raise RankFailure(self.failure() or msg)
            time.sleep(self.poll)
        if self.rank == 0 and self.step > 1:
            self.store.delete_key(f"{self.prefix}/arrived/{self.step - 1}")


def run_dist(gen, guard: Optional[StepGuard] = None):
    """Drive a step generator with torch.distributed collectives (this process = one rank).
    With a :class:`StepGuard`, the step starts with its arrival check and an exception raised
    while the step runs is posted to the other ranks before it propagates."""
    if guard is None:
        return _serve_dist(gen)
    try:
        guard.begin()
    except BaseException:
        gen.close()
        raise
    try:
        return _serve_dist(gen)
    except BaseException as e:
        if not isinstance(e, RankFailure):
            guard.fail(f"{type(e).__name__}: {e}")
        raise


def _serve_dist(gen):
    import torch.distributed as dist

    world = dist.get_world_size()
    reply = None
    while True:
        try:
            kind, arg = gen.send(reply)
        except StopIteration as e:
            return e.value
        if kind == "mark":
            if HALO_TIMER is not None and torch.cuda.is_available():
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                HALO_TIMER.append((arg, ev))
            reply = None
        elif kind == "all_gather":
            out = [torch.empty_like(arg) for _ in range(world)]
            dist.all_gather(out, arg.contiguous())
            reply = torch.stack(out)
        elif kind == "all_reduce_sum":
            reply = arg.clone()
            dist.all_reduce(reply)
        elif kind == "all_to_all":
            rows, counts, rcounts = arg
            if rcounts is None:
                sc = torch.tensor(counts, dtype=torch.int64, device=rows.device)
                rc = torch.empty_like(sc)
                dist.all_to_all_single(rc, sc)
                rcounts = [int(x) for x in rc.tolist()]
            recv = torch.empty((sum(rcounts),) + tuple(rows.shape[1:]), dtype=rows.dtype, device=rows.device)
            dist.all_to_all_single(recv, rows.contiguous(), rcounts, counts)
            reply = (recv, rcounts)
        else:
            raise ValueError(kind)


def run_local(gens: List):
    """Drive the step generators of all ranks in one process; returns their results."""
    world = len(gens)
    results = [None] * world
    pending = [None] * world
    done = [False] * world

    def advance(r, value):
        try:
            pending[r] = gens[r].send(value)
        except StopIteration as e:
            results[r] = e.value
            pending[r] = None
            done[r] = True

    for r in range(world):
        advance(r, None)
    while not all(done):
        if any(done):
            raise RuntimeError("ranks diverged: some finished while others wait in a collective")
        kinds = {p[0] for p in pending}
        if len(kinds) != 1:
            raise RuntimeError(f"collective mismatch across ranks: {sorted(kinds)}")
        kind = pending[0][0]
        args = [p[1] for p in pending]
        if kind == "mark":
            replies = [None] * world
        elif kind == "all_gather":
            t = torch.stack(args)
            replies = [t.clone() for _ in range(world)]
        elif kind == "all_reduce_sum":
            s = torch.stack(args).sum(0)
            replies = [s.clone() for _ in range(world)]
        elif kind == "all_to_all":
            chunks = []
            for rows, counts, _ in args:
                offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
                chunks.append([rows[offs[d]:offs[d + 1]] for d in range(world)])
            replies = []
            for d in range(world):
                parts = [chunks[s_][d] for s_ in range(world)]
                replies.append((torch.cat(parts), [int(p.shape[0]) for p in parts]))
        else:
            raise ValueError(kind)
        for r in range(world):
            advance(r, replies[r])
    return results


# ---------------------------------------------------------------------------- per-rank state
@dataclass
class HaloPlan:
    """What one rank sent and received in the position halo exchange of one step."""

    send_idx: torch.Tensor          # (S,) owned atom index of every row sent, grouped by destination
    send_counts: List[int]
    recv_counts: List[int]
    ghost_pos: torch.Tensor         # (G, 3) float64 image positions of the received ghosts
    ghost_species: torch.Tensor     # (G,)


def select_ghosts(dec: Decomposition, rank: int, pos: torch.Tensor, bboxes: torch.Tensor, chunk: int = 1 << 18):
    """Rows this rank sends: (send_idx, send_image, send_counts) grouped by destination rank.

    ``bboxes`` (world, 2, 3) are the owned-atom bounding boxes of all ranks; an image
    x + S.cell is sent to rank d if it lies inside d's box grown by the halo along every split
    axis (the unsplit axes are periodic in d's local system), except the atom itself
    (S = 0) for its own rank.  Rows are ordered by destination, then image, then atom.

    The owned boxes are disjoint blocks along every split axis, so only an atom within one halo
    of its own box's faces along a split axis can lie in another rank's grown box in any image:
    those candidates (one host synchronisation) are tested against all images and ranks at once
    (a second one), in chunks that bound the temporaries."""
    dev = pos.device
    world = bboxes.shape[0]
    images = dec.images()
    if pos.shape[0] == 0:
        z = torch.zeros(0, dtype=torch.int64, device=dev)
        return z, z, [0] * world
    cell = torch.tensor(dec.cell, dtype=torch.float64, device=dev)
    split = torch.tensor(dec.split, device=dev)
    lo = bboxes[:, 0, :] - dec.halo
    hi = bboxes[:, 1, :] + dec.halo
    margin = dec.halo * (1.0 + 1e-9) + 1e-9
    near = ((pos - bboxes[rank, 0]) <= margin) | ((bboxes[rank, 1] - pos) <= margin)
    cand = (near & split).any(1).nonzero().squeeze(1)
    shifts = torch.tensor(images, dtype=torch.float64, device=dev) @ cell          # (I, 3)
    zero = images.index((0, 0, 0))
    rows_s, rows_i, rows_d = [], [], []
    for c0 in range(0, cand.shape[0], chunk):
        cc = cand[c0:c0 + chunk]
        x = pos[cc][None, :, :] + shifts[:, None, :]                               # (I, nc, 3)
        inside = ((x[:, :, None, :] >= lo[None, None]) & (x[:, :, None, :] <= hi[None, None])) | ~split
        inside = inside.all(-1)                                                    # (I, nc, world)
        inside[zero, :, rank] = False
        nz = inside.nonzero()                                                      # (image, atom, rank)
        rows_s.append(nz[:, 0])
        rows_i.append(cc[nz[:, 1]])
        rows_d.append(nz[:, 2])
    if not rows_d:
        z = torch.zeros(0, dtype=torch.int64, device=dev)
        return z, z, [0] * world
    d = torch.cat(rows_d)
    i = torch.cat(rows_i)
    s = torch.cat(rows_s)
    order = torch.sort((d * (len(images) + 1) + s) * (pos.shape[0] + 1) + i, stable=True).indices
    d, i, s = d[order], i[order], s[order]
    counts = torch.bincount(d, minlength=world).tolist()
    return i, s, counts


def halo_exchange(dec: Decomposition, rank: int, pos: torch.Tensor, species: torch.Tensor):
    """Position halo exchange of one step (a generator of collectives; returns a HaloPlan)."""
    if pos.shape[0]:
        bb = torch.stack([pos.min(0).values, pos.max(0).values])
    else:  # an empty rank's box contains nothing
        bb = torch.tensor([[np.inf] * 3, [-np.inf] * 3], dtype=torch.float64, device=pos.device)
    bboxes = yield from all_gather(bb)
    idx, img, counts = select_ghosts(dec, rank, pos, bboxes)
    cell = torch.tensor(dec.cell, dtype=torch.float64, device=pos.device)
    shifts = torch.tensor(dec.images(), dtype=torch.float64, device=pos.device) @ cell
    send_pos = pos[idx] + shifts[img]
    gpos, rcounts = yield from all_to_all(send_pos, counts)
    gspec, _ = yield from all_to_all(species[idx], counts, rcounts)
    return HaloPlan(idx, counts, rcounts, gpos, gspec)


def return_ghost_forces(plan: HaloPlan, owned_forces: torch.Tensor, ghost_forces: torch.Tensor):
    """Reverse exchange: every ghost's force goes back to its owner and is added there."""
    back, _ = yield from all_to_all(ghost_forces.contiguous(), plan.recv_counts, plan.send_counts)
    out = owned_forces.clone()
    if back.shape[0]:
        out.index_add_(0, plan.send_idx, back.to(out.dtype))
    return out


Evaluator = Callable[..., Dict[str, torch.Tensor]]


def decomposed_step(dec: Decomposition, rank: int, pos: torch.Tensor, species: torch.Tensor, evaluate: Evaluator,
                    want_virial: bool = False):
    """One energy + forces step of this rank's owned atoms ``pos`` (n, 3) float64 (a generator of
    collectives; drive it with :func:`run_dist` or :func:`run_local`).

    ``evaluate(pos_local, species_local, num_local, pbc) -> {"energy", "forces", "atom_energy"[,
    "virial"]}`` evaluates the local system (owned atoms first); its ``energy`` is the sum over
    the first ``num_local`` atoms only and its forces are ``-dE_local/dpos`` for all local atoms.
    Returns the total energy (all ranks), the owned atoms' forces and energies, and the total
    virial when asked."""
    n = pos.shape[0]
    yield from halo_mark("begin")
    plan = yield from halo_exchange(dec, rank, pos, species)
    yield from halo_mark("end")
    pos_l = torch.cat([pos, plan.ghost_pos.to(pos.dtype)])
    spec_l = torch.cat([species, plan.ghost_species.to(species.dtype)])
    counts = getattr(evaluate, "local_counts", None)
    if counts is not None:  # an evaluator that needs whole-system sums of per-rank counts
        totals = yield from all_reduce_sum(counts(pos_l, n, dec.local_pbc))
        out = evaluate(pos_l, spec_l, n, dec.local_pbc, totals=totals)
    else:
        out = evaluate(pos_l, spec_l, n, dec.local_pbc)
    f = out["forces"]
    yield from halo_mark("begin")
    forces = yield from return_ghost_forces(plan, f[:n], f[n:])
    yield from halo_mark("end")
    red = [out["energy"].reshape(1).to(torch.float64)]
    if want_virial:
        red.append(out["virial"].reshape(9).to(torch.float64))
    tot = yield from all_reduce_sum(torch.cat(red))
    res = {"energy": tot[0], "forces": forces, "atom_energy": out["atom_energy"][:n],
           "num_ghosts": int(pos_l.shape[0] - n)}
    if want_virial:
        res["virial"] = tot[1:10].reshape(3, 3)
    return res


# ---------------------------------------------------------------------------- per-layer exchange
def exchange_ghost_rows(plan: HaloPlan, rows: torch.Tensor, num_local: int):
    """Forward ghost-feature exchange (the reference's sync_after_scatter, cli/inference_ddp.py:
    191-246): every rank sends the rows of its owned atoms that are ghosts elsewhere and
    overwrites its own ghost rows ``rows[num_local:]`` with their owners' rows, in place."""
    flat = rows.reshape(rows.shape[0], -1)
    recv, _ = yield from all_to_all(flat[plan.send_idx], plan.send_counts, plan.recv_counts)
    if recv.shape[0]:
        flat[num_local:num_local + recv.shape[0]] = recv
    return rows


def return_ghost_rows(plan: HaloPlan, rows: torch.Tensor, num_local: int):
    """Adjoint of :func:`exchange_ghost_rows` on gradients: the ghost rows' gradients go back to
    their owners and are added to the owned rows; the ghost rows are then zero (a ghost's own
    value was overwritten, so nothing flows through it)."""
    flat = rows.reshape(rows.shape[0], -1)
    back, _ = yield from all_to_all(flat[num_local:].contiguous(), plan.recv_counts, plan.send_counts)
    if back.shape[0]:
        flat.index_add_(0, plan.send_idx, back)
    flat[num_local:] = 0
    return rows


def owned_receiver_graph(g, num_local: int):
    """The dst-sorted CSR graph restricted to edges whose receiver is owned (rows of ghosts empty):
    with ghost features exchanged every layer, only owned receivers are evaluated."""
    from .ictd import GraphCSR

    e_own = int(g.row_ptr[num_local].item())
    row_ptr = g.row_ptr.clone()
    row_ptr[num_local + 1:] = e_own
    src = g.src[:e_own].contiguous()
    shift = g.shift[:e_own].contiguous()
    tr_ptr, tr_eid = GraphCSR.transpose(row_ptr, src, g.num_atoms)
    order = g.order[:e_own] if g.order is not None else None
    return GraphCSR(g.num_atoms, row_ptr, src, shift, tr_ptr, tr_eid, order)


def layer_exchange_step(dec: Decomposition, rank: int, pos: torch.Tensor, species: torch.Tensor, engine,
                        cutoff: float, want_virial: bool = False):
    """One energy + forces step with a per-layer ghost-feature exchange (a generator of
    collectives, like :func:`decomposed_step`), for the ictd and the sparse engine: the halo
    ``dec.halo`` needs to cover one cutoff only.  The local graph holds the edges into owned
    atoms; after each interaction layer whose features a later layer reads, the ghost rows are
    overwritten by their owners' rows; in the reverse pass the ghost rows' gradients go back to
    their owners before the layer that produced them runs backward; the ghost forces (edge
    endpoints) go back as in :func:`decomposed_step`.  Energies and virials are summed over ranks.
    The sparse model's conv2 normaliser is the whole system's E / N (edges into owned atoms and
    owned atoms, summed over ranks), as the reference computes it on the whole graph."""
    from .neighbors import build_graph
    from .sparse import SparseEngine

    n = pos.shape[0]
    dev = pos.device
    nint = engine.cfg.num_interaction
    yield from halo_mark("begin")
    plan = yield from halo_exchange(dec, rank, pos, species)
    yield from halo_mark("end")
    pos_l = torch.cat([pos, plan.ghost_pos.to(pos.dtype)])
    spec_l = torch.cat([species, plan.ghost_species.to(species.dtype)])
    n_all = int(pos_l.shape[0])
    cell_t = torch.as_tensor(dec.cell, dtype=torch.float64, device=dev).reshape(1, 3, 3)
    g = owned_receiver_graph(build_graph(pos_l, cell_t, cutoff, pbc=dec.local_pbc, transpose=False), n)
    batch = torch.zeros(n_all, dtype=torch.int32, device=dev)
    if isinstance(engine, SparseEngine):
        counts = torch.stack([g.row_ptr[n].to(torch.float64),
                              torch.tensor(float(n), dtype=torch.float64, device=dev)])
        totals = yield from all_reduce_sum(counts)
        avg = max(float(totals[0]) / max(float(totals[1]), 1.0), 1e-8)
        engine.begin_steps(pos_l, spec_l, batch, cell_t, g, num_local=n, avg_num_neighbors=avg)
    else:
        # every layer on all rows (ghost rows have no edges and are overwritten), the readout on the owned
        engine.begin_steps(pos_l, spec_l, batch, cell_t, g, num_local=n, layer_atoms=[n_all] * (nint - 1) + [n])
    for k in range(nint - 1):
        feats = engine.forward_step(k)
        yield from halo_mark("begin")
        yield from exchange_ghost_rows(plan, feats, n)
        yield from halo_mark("end")
    engine.forward_step(nint - 1)  # read by the readout only
    energy, atom_e = engine.forward_step(nint)
    out = engine.begin_backward(want_virial=want_virial)
    engine.backward_step(nint)
    for k in range(nint - 1, -1, -1):
        if k < nint - 1:
            yield from halo_mark("begin")
            yield from return_ghost_rows(plan, engine.feature_buffer(1, k), n)
            yield from halo_mark("end")
        engine.backward_step(k)
    f = out["forces"]
    yield from halo_mark("begin")
    forces = yield from return_ghost_forces(plan, f[:n], f[n:])
    yield from halo_mark("end")
    red = [energy.reshape(1).to(torch.float64)]
    if want_virial:
        red.append(out["virial"].reshape(9).to(torch.float64))
    tot = yield from all_reduce_sum(torch.cat(red))
    res = {"energy": tot[0], "forces": forces, "atom_energy": atom_e[:n], "num_ghosts": n_all - n,
           "num_edges": g.num_edges}
    if want_virial:
        res["virial"] = tot[1:10].reshape(3, 3)
    return res


SHELL_MARGIN = 1e-3  # relative: covers float32 rounding of edge lengths at ~1000 A coordinates


def layer_shells(pos: torch.Tensor, num_local: int, split: Sequence[bool], cutoff: float, num_interaction: int):
    """Receptive-field order of a local system [owned | ghosts] for the engine's ``layer_atoms``.

    ``d(x)`` = Euclidean distance of ``x`` from the owned atoms' bounding box along the split
    axes (the others are periodic in the local system), ``shell(x) = ceil(d / w)`` with
    ``w = cutoff (1 + SHELL_MARGIN)``.  An edge is shorter than the cutoff, so the sender of a
    receiver in shell ``s`` lies in shell ``<= s + 1`` even after float32 rounding of the edge
    length.  Owned energies need layer k (conv1 = 0) only on shells ``<= nint - 1 - k`` and
    positions only on shells ``<= nint``; every sender that an evaluated receiver reads was
    evaluated one layer earlier.

    Returns ``(perm, layer_atoms)``: ``perm`` indexes ``pos`` — owned atoms first in their order,
    then the ghosts of shells ``<= nint`` stably sorted by shell (farther ghosts are dropped) —
    and ``layer_atoms[k]`` = number of leading atoms of ``perm`` in shells ``<= nint - 1 - k``."""
    n = int(pos.shape[0])
    dev = pos.device
    nint = int(num_interaction)
    own = torch.arange(num_local, device=dev)
    if n == num_local or num_local == 0:
        return torch.arange(n, device=dev), [n] * nint
    p = pos.to(torch.float64)
    lo = p[:num_local].min(0).values
    hi = p[:num_local].max(0).values
    g = p[num_local:]
    over = torch.clamp(torch.maximum(lo - g, g - hi), min=0.0)
    over = over * torch.tensor([1.0 if s else 0.0 for s in split], dtype=torch.float64, device=dev)
    d = torch.linalg.vector_norm(over, dim=1)
    w = float(cutoff) * (1.0 + SHELL_MARGIN)
    shell = torch.ceil(d / w).to(torch.int64)
    keep = (shell <= nint).nonzero().squeeze(1)
    order = torch.sort(shell[keep], stable=True)
    ghosts = keep[order.indices] + num_local
    perm = torch.cat([own, ghosts])
    counts = torch.bincount(order.values, minlength=nint + 1)[: nint + 1]
    cum = (num_local + torch.cumsum(counts, 0)).tolist()   # atoms in shells <= s
    return perm, [int(cum[nint - 1 - k]) for k in range(nint)]


def ictd_evaluator(engine, cell, cutoff: float, want_virial: bool = False, restrict_layers: bool = True) -> Evaluator:
    """Evaluator of :func:`decomposed_step` backed by the native engine (one GPU per rank):
    GPU cell-list neighbour list of the local system, forward with ``num_local`` (owned atoms),
    reverse pass for the forces (and the virial).

    With ``restrict_layers`` the ghosts are ordered by distance shell (:func:`layer_shells`) and
    the engine evaluates interaction layer k only on the receivers within ``nint - 1 - k`` shells
    of the owned atoms (the readout on owned atoms only); ghosts beyond ``nint`` shells are not
    used.  The owned energies and all forces are unchanged (the dropped work only fed ghost
    energies, which carry no weight)."""
    from .neighbors import build_graph

    dev = engine.device
    cell_t = torch.as_tensor(np.asarray(cell), dtype=torch.float64, device=dev).reshape(1, 3, 3)
    nint = engine.cfg.num_interaction
    batch_cache = {}

    def evaluate(pos, species, num_local, pbc):
        n_all = int(pos.shape[0])
        layers = None
        if restrict_layers:
            perm, layers = layer_shells(pos, num_local, [not p for p in pbc], cutoff, nint)
            pos, species = pos[perm], species[perm]
        g = build_graph(pos, cell_t, cutoff, pbc=pbc)
        n = int(pos.shape[0])
        if n not in batch_cache:
            batch_cache.clear()
            batch_cache[n] = torch.zeros(n, dtype=torch.int32, device=dev)
        energy, atom_e = engine.forward(pos, species, batch_cache[n], cell_t, g, num_local=num_local,
                                        layer_atoms=layers)
        out = engine.backward(want_virial=want_virial)
        forces = out["forces"]
        if restrict_layers:
            full_f = torch.zeros(n_all, 3, dtype=forces.dtype, device=dev)
            full_f[perm] = forces
            full_e = torch.zeros(n_all, dtype=atom_e.dtype, device=dev)
            full_e[perm] = atom_e
            forces, atom_e = full_f, full_e
        res = {"energy": energy[0], "forces": forces, "atom_energy": atom_e}
        if want_virial:
            res["virial"] = out["virial"][0]
        return res

    return evaluate


def sparse_evaluator(engine, cell, cutoff: float, want_virial: bool = False) -> Evaluator:
    """Evaluator of :func:`decomposed_step` backed by the native pure-cartesian-sparse engine:
    GPU cell-list neighbour list of the local system, forward with ``num_local`` (owned atoms'
    energies), reverse pass for the forces (and the virial).  Every layer runs on all local atoms
    (the sparse engine has no receptive-field restriction); the owned energies are exact because
    the halo covers the receptive field.

    The reference's conv2 divides by E / N of the graph it is given
    (``pure_cartesian_sparse_layers.py:418``); a rank's local graph has truncated neighbour lists
    at the halo's edge, so the evaluator asks :func:`decomposed_step` for the whole system's
    E / N: ``local_counts`` gives (edges into owned atoms, owned atoms), summed over ranks."""
    from .neighbors import build_graph

    dev = engine.device
    cell_t = torch.as_tensor(np.asarray(cell), dtype=torch.float64, device=dev).reshape(1, 3, 3)
    batch_cache = {}
    graph = {}

    def local_counts(pos, num_local, pbc):
        g = build_graph(pos, cell_t, cutoff, pbc=pbc)
        graph["g"], graph["key"] = g, (pos.data_ptr(), int(pos.shape[0]))
        e_owned = g.row_ptr[num_local].to(torch.float64)  # edges are sorted by receiver, owned first
        return torch.stack([e_owned, torch.tensor(float(num_local), dtype=torch.float64, device=e_owned.device)])

    def evaluate(pos, species, num_local, pbc, totals=None):
        if graph.get("key") == (pos.data_ptr(), int(pos.shape[0])):
            g = graph.pop("g")
            graph.pop("key")
        else:
            g = build_graph(pos, cell_t, cutoff, pbc=pbc)
        n = int(pos.shape[0])
        if n not in batch_cache:
            batch_cache.clear()
            batch_cache[n] = torch.zeros(n, dtype=torch.int32, device=dev)
        avg = None
        if totals is not None:
            avg = max(float(totals[0]) / max(float(totals[1]), 1.0), 1e-8)
        energy, atom_e = engine.forward(pos, species, batch_cache[n], cell_t, g, num_local=num_local,
                                        avg_num_neighbors=avg)
        out = engine.backward(want_virial=want_virial)
        res = {"energy": energy[0], "forces": out["forces"], "atom_energy": atom_e}
        if want_virial:
            res["virial"] = out["virial"][0]
        return res

    evaluate.local_counts = local_counts
    return evaluate
