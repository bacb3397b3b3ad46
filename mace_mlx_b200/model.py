"""Host engine of the B200 MACE step.

``MACEModel`` loads a converted model directory (the reference's
``config.json`` + ``weights.npz``, ``model.py:664-720``), packs it once, and
drives ``libmace_b200`` through its C ABI.  torch is used only to own device
memory and streams; every computation of the step runs in the library's
kernels.
"""

from __future__ import annotations

import dataclasses

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np
import torch

from . import native as nv
from .pack import PackedModel
from .spec import ModelSpec
from .weights import check_weights, load_model_dir


class _CudaArray:
    """Zero-copy view of a device buffer owned by the library."""

    def __init__(self, ptr: int, n: int, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {
            "shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 2, "strides": None,
        }


@dataclass
class EdgeSet:
    """Receiver-sorted directed edges on the device (output of the GPU neighbour list)."""

    sender: torch.Tensor  # (cap,) int32
    receiver: torch.Tensor  # (cap,) int32
    shifts: torch.Tensor  # (cap, 3) int32
    row_ptr: torch.Tensor  # (N+1,) int32
    rev: torch.Tensor  # (cap,) int32
    n_edges: int
    _chunks: dict = dataclasses.field(default_factory=dict, repr=False)

    def receiver_chunks(self, max_edges: int) -> tuple[np.ndarray, np.ndarray]:
        """Receiver ranges whose edge counts stay <= max_edges (host int64 arrays).

        Returns (nodes, edges): boundaries 0 .. N and row_ptr at them.  Cached,
        so the arrays (and the pointers the library sees) stay the same while
        the list is unchanged.
        """
        if max_edges not in self._chunks:
            rp = self.row_ptr.cpu().numpy().astype(np.int64)
            n = rp.shape[0] - 1
            nodes = [0]
            while nodes[-1] < n:
                start = nodes[-1]
                # last receiver boundary with row_ptr <= row_ptr[start] + max_edges
                end = int(np.searchsorted(rp, rp[start] + max_edges, side="right")) - 1
                if end <= start:
                    raise ValueError(f"receiver {start} alone has more than {max_edges} edges")
                nodes.append(min(end, n))
            nodes_a = np.asarray(nodes, dtype=np.int64)
            self._chunks[max_edges] = (nodes_a, np.ascontiguousarray(rp[nodes_a]))
        return self._chunks[max_edges]

    def numpy(self):
        e = self.n_edges
        return (self.sender[:e].cpu().numpy(), self.receiver[:e].cpu().numpy(),
                self.shifts[:e].cpu().numpy())


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


class MACEModel:
    def __init__(self, model_dir: str | os.PathLike | None = None, *, config: dict | None = None,
                 weights: dict | None = None, device: int | str | torch.device = 0, head: str | None = None):
        """``head``: the head of a multi-head model whose energies are computed
        (default: the first); an unknown name raises ``ValueError``."""
        if model_dir is not None:
            config, weights = load_model_dir(model_dir)
        if config is None or weights is None:
            raise ValueError("give a model directory or (config, weights)")
        self.config = config
        self.spec = ModelSpec.from_config(config, head=head)
        self.heads = self.spec.heads
        self.head = self.spec.heads[self.spec.head_idx]
        check_weights(self.spec, weights)
        dev = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
        if dev.type != "cuda":
            raise ValueError("MACEModel runs on a CUDA device only")
        if not torch.cuda.is_available():
            raise RuntimeError("no CUDA device available: the B200 step has no CPU fallback")
        self.device = torch.device("cuda", dev.index if dev.index is not None else torch.cuda.current_device())
        self.lib = nv.load_library()
        self.packed = PackedModel(self.spec, weights)
        ctx = C.c_void_p()
        nv.check(self.lib.mace_ctx_create(C.byref(self.packed.desc), self.device.index, C.byref(ctx)), self.lib)
        self.ctx = ctx
        self.z_table = self.spec.z_table
        self.r_max = self.spec.r_max
        self._cap = (0, 0, 0)
        self._edge_cap = 0
        # per-edge radial-weight buffers (all layers' w and MLP activations, one dw)
        per_edge = 0
        for lay in self.spec.layers:
            w = lay.mlp_widths
            per_edge += w[-1] + sum(w[1:-1])
        per_edge += max(lay.mlp_widths[-1] for lay in self.spec.layers)
        self.bytes_per_chunk_edge = 4 * per_edge
        # MACE_B200_CHUNK_BYTES caps the radial-weight buffers; by default they
        # take up to 80% of the device memory left after the rest of the workspace
        env = os.environ.get("MACE_B200_CHUNK_BYTES")
        self._chunk_budget = float(env) if env else None
        self.max_chunk_edges = max(4096, int(self._chunk_budget // self.bytes_per_chunk_edge)) if env else 1 << 40

    def close(self):
        if getattr(self, "ctx", None) is not None and self.ctx.value:
            self.lib.mace_ctx_destroy(self.ctx)
            self.ctx = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------
    def species_index(self, numbers) -> np.ndarray:
        """Atomic numbers -> model element indices (raises for unsupported Z)."""
        numbers = np.asarray(numbers, dtype=np.int64)
        if self.z_table is None:
            idx = numbers.copy()
            ok = (idx >= 0) & (idx < self.spec.num_elements)
        else:
            lut = np.full(max(max(self.z_table), int(numbers.max(initial=0))) + 1, -1, dtype=np.int64)
            lut[np.asarray(self.z_table)] = np.arange(len(self.z_table))
            idx = lut[numbers]
            ok = idx >= 0
        if not np.all(ok):
            bad = int(numbers[~ok][0])
            supported = sorted(self.z_table) if self.z_table is not None else list(range(self.spec.num_elements))
            raise ValueError(f"Atomic number {bad} is not supported by this model. Supported: {supported}")
        return idx.astype(np.int32)

    def reserve(self, n_nodes: int, n_edges: int) -> None:
        """Workspace for n_nodes / n_edges; radial-weight buffers for at most max_chunk_edges."""
        if n_nodes <= self._cap[0] and n_edges <= self._cap[1] and min(n_edges, self.max_chunk_edges) <= self._cap[2]:
            return
        N = max(n_nodes, self._cap[0])
        E = max(n_edges, self._cap[1])
        if self._chunk_budget is None:
            # size the rest of the workspace first, then give the radial buffers what is left
            small = min(E, 4096)
            nv.check(self.lib.mace_ctx_reserve_chunked(self.ctx, N, E, small), self.lib)
            self._cap = (N, E, small)
            free, _ = torch.cuda.mem_get_info(self.device)
            self.max_chunk_edges = max(4096, int(0.8 * free // self.bytes_per_chunk_edge))
        EC = max(min(E, self.max_chunk_edges), self._cap[2])
        nv.check(self.lib.mace_ctx_reserve_chunked(self.ctx, N, E, EC), self.lib)
        self._cap = (N, E, EC)

    def workspace_bytes(self) -> int:
        b = C.c_int64()
        nv.check(self.lib.mace_ctx_workspace_bytes(self.ctx, C.byref(b)), self.lib)
        return b.value

    # ------------------------------------------------------------------
    def neighbour_list(self, pos64: torch.Tensor, cell64: torch.Tensor | None, pbc, graph_ptr: torch.Tensor,
                       r_cut: float, edges: EdgeSet | None = None) -> EdgeSet:
        """GPU "ijS" list (cutoff r_cut) for positions already on the device."""
        n = pos64.shape[0]
        self.reserve(n, self._cap[1])
        pbc_arr = (C.c_int32 * 3)(*[int(bool(x)) for x in pbc])
        stream = torch.cuda.current_stream(self.device).cuda_stream
        cap = edges.sender.shape[0] if edges is not None and edges.row_ptr.shape[0] == n + 1 else 0
        if cap == 0:
            cap = max(1024, int(n * 64))
        for _ in range(3):
            if edges is None or edges.sender.shape[0] < cap or edges.row_ptr.shape[0] != n + 1:
                i32 = dict(dtype=torch.int32, device=self.device)
                edges = EdgeSet(torch.empty(cap, **i32), torch.empty(cap, **i32), torch.empty(cap, 3, **i32),
                                torch.empty(n + 1, **i32), torch.empty(cap, **i32), 0)
            ne = C.c_int64()
            rc = self.lib.mace_nl_build(
                self.ctx, pos64.data_ptr(), _ptr(cell64), pbc_arr, graph_ptr.data_ptr(), graph_ptr.shape[0] - 1,
                n, float(r_cut), edges.sender.data_ptr(), edges.receiver.data_ptr(), edges.shifts.data_ptr(),
                edges.row_ptr.data_ptr(), edges.rev.data_ptr(), edges.sender.shape[0], C.byref(ne), stream)
            if rc == nv.MACE_ERR_NL_OVERFLOW:
                cap = int(ne.value * 1.25) + 1024
                edges = None
                continue
            nv.check(rc, self.lib)
            edges.n_edges = int(ne.value)
            edges._chunks.clear()
            return edges
        raise RuntimeError("neighbour list did not fit after resizing")

    # ------------------------------------------------------------------
    def evaluate(self, pos: torch.Tensor, cell: torch.Tensor | None, species: torch.Tensor,
                 graph_ptr: torch.Tensor, edges: EdgeSet, *, forces: bool = True, virial: bool = False,
                 out: dict | None = None, graph: bool = False, energy_weight: torch.Tensor | None = None,
                 halo=None, halo_exchange=None, active: tuple[int, int] | None = None) -> dict:
        """Energy per graph (float64), node energies, forces and the raw virial.

        All inputs are device tensors: pos (N,3) float32, cell (3,3) float32 or
        None, species (N,) int32 model indices, graph_ptr (G+1,) int32.
        Asynchronous on the current stream.  ``graph=True`` replays the step as
        a CUDA graph (re-captured whenever a buffer address or size changes).
        ``energy_weight`` (N,) float32 weighs each node's energy in the graph
        energies and all gradients (owned 1 / ghost 0 under domain decomposition).
        Lists with more than ``max_chunk_edges`` edges run the radial work in
        receiver chunks (the MLP of each chunk is recomputed in the backward).
        ``halo(phase, layer, rows)`` is called between layers with the (N, row)
        node-feature (phase 0) or feature-gradient (phase 1) rows, on the step's
        stream (domain decomposition; see mace_halo_fn in include/mace_b200.h).
        ``halo_exchange`` (a ``distributed.NativeHaloExchange``) does the same
        inside the library, graph replay included.  ``active = (n, e)`` makes
        nodes [0, n) the only receivers (their edges are [0, e)); later nodes
        are senders only (ghost atoms, energy weight 0).
        """
        N = pos.shape[0]
        E = edges.n_edges
        self.reserve(N, E)
        G = graph_ptr.shape[0] - 1
        if out is None:
            out = {
                "energy": torch.empty(G, dtype=torch.float64, device=self.device),
                "node_energy": torch.empty(N, dtype=torch.float32, device=self.device),
                "forces": torch.empty(N, 3, dtype=torch.float32, device=self.device) if forces else None,
                "virial": torch.empty(9, dtype=torch.float64, device=self.device) if virial else None,
            }
        sysd = nv.System(
            n_nodes=N, n_edges=E, num_graphs=G, pos=pos.data_ptr(), cell=_ptr(cell),
            species=species.data_ptr(), graph_ptr=graph_ptr.data_ptr(), sender=edges.sender.data_ptr(),
            receiver=edges.receiver.data_ptr(), shifts=edges.shifts.data_ptr(), row_ptr=edges.row_ptr.data_ptr(),
            rev=edges.rev.data_ptr(), energy_weight=_ptr(energy_weight))
        if active is not None and E <= self.max_chunk_edges:
            # (a list split into radial chunks keeps every receiver: the per-edge
            # sender terms that inactive receivers rely on need a one-chunk list)
            sysd.n_active, sysd.e_active = int(active[0]), int(active[1])
        if halo_exchange is not None:
            sysd.halo_exchange = halo_exchange.handle
        if halo is not None:
            dev = self.device

            def _cb(user, phase, layer, ptr, row_len, stream):
                try:
                    rows = torch.as_tensor(_CudaArray(ptr, N * row_len), device=dev).view(N, row_len)
                    # a NULL stream (the legacy default stream) arrives as None
                    st = torch.cuda.ExternalStream(stream, device=dev) if stream else torch.cuda.default_stream(dev)
                    with torch.cuda.stream(st):
                        halo(int(phase), int(layer), rows)
                    return 0
                except Exception as e:  # noqa: BLE001  (reported through the status code)
                    self.halo_error = e
                    return 1

            self._halo_fn = nv.HaloFn(_cb)  # kept alive for the duration of the call
            sysd.halo = C.cast(self._halo_fn, C.c_void_p)
            graph = False
        if E > self.max_chunk_edges:
            nodes, ebounds = edges.receiver_chunks(self.max_chunk_edges)
            sysd.n_chunks = len(nodes) - 1
            sysd.chunk_nodes = nodes.ctypes.data
            sysd.chunk_edges = ebounds.ctypes.data
        outs = nv.Outputs(energy=_ptr(out["energy"]), node_energy=_ptr(out["node_energy"]),
                          forces=_ptr(out.get("forces")), virial=_ptr(out.get("virial")))
        flags = (nv.WANT_FORCES if forces else 0) | (nv.WANT_VIRIAL if virial else 0) | (nv.USE_GRAPH if graph else 0)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        self.halo_error = None
        rc = self.lib.mace_forward_backward(self.ctx, C.byref(sysd), C.byref(outs), flags, stream)
        if rc and self.halo_error is not None:
            raise RuntimeError("halo exchange callback failed") from self.halo_error
        nv.check(rc, self.lib)
        return out

    def last_launch_count(self) -> int:
        c = C.c_int32()
        nv.check(self.lib.mace_last_launch_count(self.ctx, C.byref(c)), self.lib)
        return c.value

    def profile_enable(self, enable: bool = True) -> None:
        nv.check(self.lib.mace_profile_enable(self.ctx, int(enable)), self.lib)

    def profile_read(self) -> list[dict]:
        """Per (kernel, layer) launch counts and total event-timed milliseconds."""
        mx = 128
        names = C.create_string_buffer(32 * mx)
        layers = (C.c_int32 * mx)()
        counts = (C.c_int32 * mx)()
        ms = (C.c_double * mx)()
        n = C.c_int32()
        nv.check(self.lib.mace_profile_read(self.ctx, mx, names, layers, counts, ms, C.byref(n)), self.lib)
        out = []
        for i in range(n.value):
            nm = names.raw[32 * i: 32 * (i + 1)].split(b"\0", 1)[0].decode()
            out.append({"name": nm, "layer": layers[i], "count": counts[i], "ms": ms[i]})
        return out

    def profile_timeline(self) -> list[dict]:
        """The last profiled step's launches: name, layer, stream, start/end ms from its first launch."""
        mx = 256
        names = C.create_string_buffer(32 * mx)
        layers = (C.c_int32 * mx)()
        streams = (C.c_int32 * mx)()
        t0 = (C.c_float * mx)()
        t1 = (C.c_float * mx)()
        n = C.c_int32()
        nv.check(self.lib.mace_profile_timeline(self.ctx, mx, names, layers, streams, t0, t1, C.byref(n)),
                 self.lib)
        return [{"name": names.raw[32 * i: 32 * (i + 1)].split(b"\0", 1)[0].decode(), "layer": layers[i],
                 "stream": streams[i], "start_ms": t0[i], "end_ms": t1[i]} for i in range(n.value)]

    def error_flag(self) -> int:
        c = C.c_int32()
        nv.check(self.lib.mace_ctx_error_flag(self.ctx, C.byref(c)), self.lib)
        return c.value

    def debug_buffer(self, stage: str, layer: int | None = None) -> torch.Tensor:
        """Copy of an internal per-stage buffer of the last evaluation (parity tests).

        The radial weights (stage "w") come back in the kernels' 128-edge tile
        layout; ``edge_tiles_to_rows`` turns them into an (E, W) matrix.
        """
        bid = 15 * 16 + nv.EDGE_STAGES[stage] if layer is None else layer * 16 + nv.STAGES[stage]
        ptr, n = C.c_void_p(), C.c_int64()
        nv.check(self.lib.mace_debug_buffer(self.ctx, bid, C.byref(ptr), C.byref(n)), self.lib)
        if not ptr.value or n.value == 0:
            return torch.empty(0, device=self.device)
        torch.cuda.synchronize(self.device)
        return torch.as_tensor(_CudaArray(ptr.value, n.value), device=self.device).clone()


def edge_tiles_to_rows(buf: torch.Tensor, n_edges: int, width: int) -> torch.Tensor:
    """(E, W) view of a per-edge matrix stored in 128-edge tiles.

    Tile e // 128 holds ceil(W / 32) chunks of 128 rows x 32 floats; column c
    of edge e is in chunk c // 32, row e % 128, at 16-byte group
    ((c % 32) // 4) ^ (e % 8), position c % 4 (the 128B-swizzled operand
    layout of the tensor-core MLP kernels).
    """
    nch = -(-width // 32)
    nt = -(-n_edges // 128)
    x = buf[: nt * nch * 4096].reshape(nt, nch, 128, 8, 4)
    rows = torch.arange(128, device=buf.device)
    groups = torch.arange(8, device=buf.device)
    src = groups[None, :] ^ (rows[:, None] & 7)
    x = x[:, :, rows[:, None], src, :]
    return x.permute(0, 2, 1, 3, 4).reshape(nt * 128, nch * 32)[:n_edges, :width]
