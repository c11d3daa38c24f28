"""GPU neighbour list with the semantics of ``radius_graph_pbc_gpu`` (``utils/graph_utils.py:192-258``).

``build_graph`` runs the native count + fill (cell list for large periodic orthorhombic
frames, all-pairs otherwise; identical edge sets, float64 distance test in a fixed order)
and the transpose CSR, returning a ``GraphCSR`` ready for ``ICTDEngine``.
``radius_graph_pbc`` returns the flat ``(edge_src, edge_dst, edge_shifts)`` triple of the
reference function (canonical order: dst, then src, then shift).

``max_num_neighbors`` applies the reference's per-source cap (``graph_utils.py:192, 240``): its
torch_cluster search runs once per image shift and keeps, for every source atom, the first
``max_num_neighbors`` candidates in ascending index order, the self pair at zero shift taking a
slot.  ``radius_graph_pbc`` defaults to the reference's 100; ``build_graph`` to no cap.
"""

from __future__ import annotations

from typing import Sequence

import numpy as np
import torch

from fsctep_b200 import _native as N
from fsctep_b200.ictd import GraphCSR


def _sidx_to_shift(sidx: torch.Tensor) -> torch.Tensor:
    s = sidx.to(torch.int32)
    return torch.stack([s // 9 - 1, (s // 3) % 3 - 1, s % 3 - 1], dim=1)


def build_graph(pos: torch.Tensor, cell: torch.Tensor, cutoff: float, frame_ptr: Sequence[int] = None,
                pbc=(True, True, True), max_num_neighbors: int = None, transpose: bool = True) -> GraphCSR:
    """pos (N,3) and cell (F,3,3) on the GPU (float64 used for the distance test).  With
    ``transpose=False`` the transpose CSR is left out (``tr_ptr`` / ``tr_eid`` None), for a caller
    that restricts the graph first."""
    dev = pos.device
    pos64 = pos.detach().to(torch.float64).contiguous()
    cell64 = cell.detach().to(device=dev, dtype=torch.float64).reshape(-1, 3, 3).contiguous()
    n = int(pos64.shape[0])
    F = int(cell64.shape[0])
    if frame_ptr is None:
        if F != 1:
            raise ValueError("frame_ptr is required with more than one cell")
        frame_ptr = [0, n]
    fp = np.ascontiguousarray(np.asarray(frame_ptr, dtype=np.int64))
    pbc_h = np.ascontiguousarray(np.asarray([1 if p else 0 for p in pbc], dtype=np.int32))
    L = N.lib()
    st = N.stream_ptr(dev)
    row_ptr = torch.empty(n + 1, dtype=torch.int32, device=dev)
    ws = torch.empty(L.fsc_neighbor_workspace_bytes(n, 0), dtype=torch.uint8, device=dev)
    ne = N.I64(0)
    N.check(L.fsc_neighbor_count(N.ptr(pos64), N.ptr(cell64), fp.ctypes.data_as(N.P), F, n,
                                 pbc_h.ctypes.data_as(N.P), float(cutoff), N.ptr(row_ptr), N.C.byref(ne),
                                 N.ptr(ws), ws.numel(), st), "fsc_neighbor_count")
    E = int(ne.value)
    src = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
    sidx = torch.empty(max(E, 1), dtype=torch.int8, device=dev)
    need = L.fsc_neighbor_workspace_bytes(n, E)
    if ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
    N.check(L.fsc_neighbor_fill(N.ptr(pos64), N.ptr(cell64), fp.ctypes.data_as(N.P), F, n,
                                pbc_h.ctypes.data_as(N.P), float(cutoff), N.ptr(row_ptr), N.ptr(src), N.ptr(sidx), E,
                                N.ptr(ws), ws.numel(), st), "fsc_neighbor_fill")
    src, sidx = src[:E], sidx[:E]
    tr_ptr = tr_eid = None
    if max_num_neighbors is not None:
        t_ptr, t_eid = GraphCSR.transpose(row_ptr, src, n)
        row_ptr, src, sidx = _cap(row_ptr, src, sidx, t_ptr, t_eid, n, int(max_num_neighbors))
    if transpose:
        tr_ptr, tr_eid = GraphCSR.transpose(row_ptr, src, n)
    shift = _sidx_to_shift(sidx).to(torch.float32).contiguous()
    g = GraphCSR(n, row_ptr, src, shift, tr_ptr, tr_eid)
    g.sidx = sidx
    return g


def _cap(row_ptr, src, sidx, tr_ptr, tr_eid, n: int, cap: int):
    L = N.lib()
    dev = src.device
    E = int(src.shape[0])
    out_ptr = torch.empty(n + 1, dtype=torch.int32, device=dev)
    out_src = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
    out_sidx = torch.empty(max(E, 1), dtype=torch.int8, device=dev)
    ws = torch.empty(L.fsc_neighbor_cap_workspace_bytes(n, E), dtype=torch.uint8, device=dev)
    ne = N.I64(0)
    N.check(L.fsc_neighbor_cap(N.ptr(row_ptr), N.ptr(src), N.ptr(sidx), n, E, N.ptr(tr_ptr), N.ptr(tr_eid), cap,
                               N.ptr(out_ptr), N.ptr(out_src), N.ptr(out_sidx), N.C.byref(ne), N.ptr(ws), ws.numel(),
                               N.stream_ptr(dev)), "fsc_neighbor_cap")
    E2 = int(ne.value)
    return out_ptr, out_src[:E2], out_sidx[:E2]


def radius_graph_pbc(pos: torch.Tensor, r: float, cell: torch.Tensor, max_num_neighbors: int = 100, pbc=None,
                     frame_ptr=None):
    """(edge_src, edge_dst, edge_shifts) like the reference, canonical order, int64 / float64;
    the argument order of ``radius_graph_pbc_gpu(pos, r, cell, max_num_neighbors=100, pbc=None)``."""
    if pbc is None:
        pbc = (True, True, True)
    g = build_graph(pos, cell, r, frame_ptr, pbc, max_num_neighbors)
    dev = pos.device
    counts = (g.row_ptr[1:] - g.row_ptr[:-1]).to(torch.int64)
    dst = torch.repeat_interleave(torch.arange(g.num_atoms, device=dev), counts)
    return g.src.to(torch.int64), dst, _sidx_to_shift(g.sidx).to(torch.float64)
