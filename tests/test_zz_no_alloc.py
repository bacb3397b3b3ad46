"""mace_nl_build_noalloc: the neighbour list for callers that cannot allocate
device memory (hosts that own the whole GPU through their own memory pool, or
loops that cannot afford cudaMalloc's implicit synchronisation).  Its scratch is
a static device array instead of a context workspace; its output must be
identical to the context-based mace_nl_build, call after call.

Collected last on purpose, so a failure here never hides the other tests."""

import ctypes as C

import numpy as np
import pytest
import torch

from helpers import graph_ptr_of, make_case
from mace_mlx_b200 import native as nv
from mace_mlx_b200.model import MACEModel
from mace_mlx_b200.structures import Structure, diamond_si, molecule_batch

pytestmark = pytest.mark.gpu


def triclinic_si(seed: int) -> Structure:
    """Diamond Si64 with a sheared cell (every lattice vector off-axis)."""
    st = diamond_si(2, 0.05, seed)
    frac = st.positions @ np.linalg.inv(st.cell)
    cell = np.array([[10.86, 0.0, 0.0], [2.7, 10.2, 0.0], [-1.9, 3.1, 9.8]])
    return Structure(frac @ cell, st.numbers.copy(), cell, st.pbc.copy())


def noalloc_nl(lib, st, r_cut, cap):
    dev = torch.device("cuda", 0)
    i32 = dict(dtype=torch.int32, device=dev)
    n = len(st)
    pos = torch.tensor(st.positions, dtype=torch.float64, device=dev)
    periodic = bool(np.any(st.pbc))
    cell = torch.tensor(st.cell, dtype=torch.float64, device=dev) if periodic else None
    gp = torch.as_tensor(graph_ptr_of(st), device=dev)
    out = {k: torch.full((cap,), -7, **i32) for k in ("sender", "receiver", "rev")}
    out["shifts"] = torch.full((cap, 3), -7, **i32)
    out["row_ptr"] = torch.full((n + 1,), -7, **i32)
    ne = C.c_int64()
    pbc = (C.c_int32 * 3)(*[int(bool(x)) for x in st.pbc])
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.mace_nl_build_noalloc(pos.data_ptr(), cell.data_ptr() if cell is not None else None, pbc,
                                       gp.data_ptr(), gp.shape[0] - 1, n, float(r_cut),
                                       out["sender"].data_ptr(), out["receiver"].data_ptr(),
                                       out["shifts"].data_ptr(), out["row_ptr"].data_ptr(), out["rev"].data_ptr(),
                                       cap, C.byref(ne), stream)
    if rc == nv.MACE_ERR_NL_OVERFLOW:
        return rc, ne.value
    nv.check(rc, lib)
    e = ne.value
    return {k: (v[:e] if k != "row_ptr" else v).cpu().numpy() for k, v in out.items()}, e


CASES = {
    "si216": lambda: (diamond_si(3, 0.05, 12), 6.0),
    "molecules": lambda: (molecule_batch(10, 9), 5.0),
    # 8-atom cell of 5.43 A with a 6 A cutoff: several periodic images per pair and self-images
    "si8_multi_image": lambda: (diamond_si(1, 0.05, 13), 6.0),
    "triclinic_si64": lambda: (triclinic_si(14), 6.0),
}


@pytest.mark.parametrize("case", list(CASES))
def test_noalloc_matches_context_build_twice(case):
    lib = nv.load_library()
    st, r_cut = CASES[case]()
    config, weights, _ = make_case("small")
    model = MACEModel(config=config, weights=weights, device=0)
    dev = model.device
    ref = model.neighbour_list(torch.tensor(st.positions, dtype=torch.float64, device=dev),
                               torch.tensor(st.cell, dtype=torch.float64, device=dev) if np.any(st.pbc) else None,
                               st.pbc, torch.as_tensor(graph_ptr_of(st), device=dev), r_cut)
    E = ref.n_edges
    want = {"sender": ref.sender[:E], "receiver": ref.receiver[:E], "shifts": ref.shifts[:E],
            "row_ptr": ref.row_ptr, "rev": ref.rev[:E]}
    want = {k: v.cpu().numpy() for k, v in want.items()}
    for _ in range(2):  # the shared scratch keeps the previous call's contents
        got, e = noalloc_nl(lib, st, r_cut, E + 64)
        assert e == E
        for k in want:
            np.testing.assert_array_equal(got[k], want[k], err_msg=k)


def test_noalloc_reports_overflow_with_the_edge_count():
    lib = nv.load_library()
    st, r_cut = diamond_si(2, 0.05, 15), 6.0
    got, E = noalloc_nl(lib, st, r_cut, 100000)
    rc, ne = noalloc_nl(lib, st, r_cut, E - 1)
    assert rc == nv.MACE_ERR_NL_OVERFLOW
    assert ne == E


def test_noalloc_rejects_a_graph_above_the_per_graph_limit():
    lib = nv.load_library()
    n = nv.NOALLOC_MAX_GRAPH_ATOMS + 1
    pbc = (C.c_int32 * 3)(0, 0, 0)
    ne = C.c_int64()
    pos = torch.zeros((n, 3), dtype=torch.float64, device="cuda")
    gp = torch.tensor([0, n], dtype=torch.int32, device="cuda")
    row_ptr = torch.zeros(n + 1, dtype=torch.int32, device="cuda")
    rc = lib.mace_nl_build_noalloc(pos.data_ptr(), None, pbc, gp.data_ptr(), 1, n, 5.0, None, None, None,
                                   row_ptr.data_ptr(), None, 0, C.byref(ne), None)
    assert rc == nv.MACE_ERR_BAD_ARG
    assert "per-graph limit" in nv.last_error(lib)


def test_noalloc_rejects_systems_above_the_limit():
    lib = nv.load_library()
    n = nv.NOALLOC_MAX_ATOMS + 1
    pbc = (C.c_int32 * 3)(0, 0, 0)
    ne = C.c_int64()
    dummy = torch.zeros(8, dtype=torch.float64, device="cuda")
    rc = lib.mace_nl_build_noalloc(dummy.data_ptr(), None, pbc, dummy.data_ptr(), 1, n, 5.0, None, None, None,
                                   dummy.data_ptr(), None, 0, C.byref(ne), None)
    assert rc == nv.MACE_ERR_BAD_ARG
    assert "exceed the limit" in nv.last_error(lib)
