"""ctypes binding of ``libmace_b200.so`` (declared in ``include/mace_b200.h``).

The structures below mirror the C header field by field.  Loading fails
loudly when the library is missing: there is no CPU fallback for the step.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmace_b200.so"

MACE_OK = 0
MACE_ERR_BAD_ARG = 1
MACE_ERR_CUDA = 2
MACE_ERR_NL_OVERFLOW = 3
MACE_ERR_TIMEOUT = 4
MACE_ERR_NCCL = 5
MACE_ERR_UNSUPPORTED = 6
MACE_ERR_EDGES = 7
ABI_VERSION = 8

MAX_LAYERS = 4
MAX_IN = 4
MAX_MID = 24
MAX_SRC = 6
MAX_CORR = 3

WANT_FORCES = 1
WANT_VIRIAL = 2
USE_GRAPH = 4

# debug buffer ids: layer * 16 + stage; layer 15 holds per-edge / global buffers
STAGES = {
    "up": 0, "w": 1, "A": 2, "msg": 3, "B": 4, "h_out": 5, "dh_out": 6, "dB": 7,
    "dmsg": 8, "dA": 9, "dup": 10, "act": 11, "dh_in": 12, "msg2": 13,
}
EDGE_STAGES = {"v": 0, "Y": 1, "b": 2, "dY": 3, "db": 4, "dv": 5, "h0": 6, "e_layers": 7, "dens": 8}

i32, i64, f32 = C.c_int32, C.c_int64, C.c_float


class Slots(C.Structure):
    _fields_ = [("n", i32), ("l", i32 * MAX_IN), ("off", i32 * MAX_IN), ("dim", i32)]


class ConvSlot(C.Structure):
    _fields_ = [("l1", i32), ("l2", i32), ("l3", i32), ("src", i32), ("off", i32), ("m_off", i32),
                ("f_cg", i64)]


class LinGroup(C.Structure):
    _fields_ = [("n_src", i32), ("src", i32 * MAX_SRC), ("f_w", i64), ("f_wt", i64)]


class ScOut(C.Structure):
    _fields_ = [("L", i32), ("corr", i32), ("n_ent", i32), ("i_ent", i64), ("f_G", i64)]


class LayerDesc(C.Structure):
    _fields_ = [
        ("C", i32), ("residual", i32),
        ("in_", Slots), ("hid", Slots), ("mid", Slots), ("inter", Slots),
        ("n_skip", i32), ("skip_in", i32 * MAX_IN), ("skip_out", i32 * MAX_IN),
        ("f_skip", i64 * MAX_IN), ("f_skip_t", i64 * MAX_IN),
        ("f_up", i64 * MAX_IN), ("f_up_t", i64 * MAX_IN),
        ("n_mlp", i32), ("mlp_w", i32 * 8), ("f_mlp", i64 * 7), ("f_mlp_t", i64 * 7),
        ("f_mlp_tc", i64), ("f_mlp_tc_bwd", i64), ("f_mlp_tc_trunk", i64), ("f_mlp_tc_trunk_bwd", i64),
        ("n_mid", i32), ("m_tot", i32), ("wnumel", i32),
        ("conv", ConvSlot * MAX_MID),
        ("lin", LinGroup * MAX_IN),
        ("sc", ScOut * MAX_IN),
        ("sc_n_bwd", i32), ("i_sc_bwd", i64), ("f_sc_bwd", i64), ("sc_gen", i32),
        ("f_prod", i64 * MAX_IN), ("f_prod_t", i64 * MAX_IN),
        ("readout_nonlinear", i32), ("readout_hidden", i32),
        ("f_ro1", i64), ("f_ro2", i64),
        ("density", i32), ("f_density", i64),
    ]


class ModelDesc(C.Structure):
    _fields_ = [
        ("abi_version", i32), ("num_layers", i32), ("num_elements", i32), ("num_bessel", i32),
        ("max_ell", i32), ("poly_p", i32), ("scale_shift", i32), ("C", i32),
        ("r_max", f32), ("inv_avg_num_neighbors", f32), ("scale", f32), ("shift", f32),
        ("f_e0", i64), ("f_emb", i64), ("f_bessel", i64), ("f_sh", i64),
        ("layers", LayerDesc * MAX_LAYERS),
        ("agnesi", i32), ("agnesi_q", f32), ("agnesi_p", f32), ("agnesi_a", f32), ("f_radius_agnesi", i64),
        ("zbl", i32), ("zbl_p", i32), ("zbl_a_exp", f32), ("zbl_a_prefactor", f32),
        ("f_radius_zbl", i64), ("f_znum", i64),
        ("envelope_on_weights", i32), ("reserved0", i32),
        ("floats", C.POINTER(f32)), ("n_floats", i64),
        ("ints", C.POINTER(i32)), ("n_ints", i64),
    ]


HALO_FEATURES = 0
HALO_GRADIENTS = 1
# int (*)(void* user, int32 phase, int32 layer, float* rows, int64 row_len, void* stream)
HaloFn = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_int64, C.c_void_p)


class System(C.Structure):
    _fields_ = [
        ("n_nodes", i64), ("n_edges", i64), ("num_graphs", i32),
        ("pos", C.c_void_p), ("cell", C.c_void_p), ("species", C.c_void_p),
        ("graph_ptr", C.c_void_p), ("sender", C.c_void_p), ("receiver", C.c_void_p),
        ("shifts", C.c_void_p), ("row_ptr", C.c_void_p), ("rev", C.c_void_p),
        ("energy_weight", C.c_void_p), ("n_chunks", i32), ("chunk_nodes", C.c_void_p),
        ("chunk_edges", C.c_void_p), ("halo", C.c_void_p), ("halo_user", C.c_void_p),
        ("n_active", i64), ("e_active", i64), ("halo_exchange", C.c_void_p),
    ]


class Outputs(C.Structure):
    _fields_ = [("energy", C.c_void_p), ("node_energy", C.c_void_p), ("forces", C.c_void_p),
                ("virial", C.c_void_p)]


class NativeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"libmace_b200 error {code}: {msg}")
        self.code = code


EXPORTED = (
    "mace_last_error", "mace_ctx_create", "mace_ctx_destroy", "mace_ctx_reserve", "mace_ctx_reserve_chunked",
    "mace_ctx_workspace_bytes", "mace_nl_build", "mace_forward_backward", "mace_debug_buffer",
    "mace_last_launch_count", "mace_ctx_error_flag", "mace_profile_enable", "mace_profile_read",
    "mace_profile_timeline",
    "mace_nl_build_noalloc", "mace_fma_probe",
    "mace_halo_unique_id", "mace_halo_create", "mace_halo_plan", "mace_halo_destroy",
)
NOALLOC_MAX_ATOMS = 131072
NOALLOC_MAX_GRAPH_ATOMS = 16384

_lib = None


def load_library(path: str | Path | None = None) -> C.CDLL:
    """Load (once) and type the shared library; raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: build it with `python -m mace_mlx_b200.build` "
            "(the B200 step has no CPU fallback)"
        )
    lib = C.CDLL(str(p))
    vp = C.c_void_p
    sig = {
        "mace_last_error": ([C.c_char_p, C.c_size_t], C.c_int),
        "mace_ctx_create": ([C.POINTER(ModelDesc), C.c_int, C.POINTER(vp)], C.c_int),
        "mace_ctx_destroy": ([vp], C.c_int),
        "mace_ctx_reserve": ([vp, i64, i64], C.c_int),
        "mace_ctx_reserve_chunked": ([vp, i64, i64, i64], C.c_int),
        "mace_ctx_workspace_bytes": ([vp, C.POINTER(i64)], C.c_int),
        "mace_nl_build": ([vp, vp, vp, C.POINTER(i32), vp, i32, i64, C.c_double, vp, vp, vp, vp, vp,
                           i64, C.POINTER(i64), vp], C.c_int),
        "mace_forward_backward": ([vp, C.POINTER(System), C.POINTER(Outputs), i32, vp], C.c_int),
        "mace_debug_buffer": ([vp, i32, C.POINTER(vp), C.POINTER(i64)], C.c_int),
        "mace_last_launch_count": ([vp, C.POINTER(i32)], C.c_int),
        "mace_ctx_error_flag": ([vp, C.POINTER(i32)], C.c_int),
        "mace_nl_build_noalloc": ([vp, vp, C.POINTER(i32), vp, i32, i64, C.c_double, vp, vp, vp, vp, vp,
                                  i64, C.POINTER(i64), vp], C.c_int),
        "mace_fma_probe": ([vp, i32, i32, vp], C.c_int),
        "mace_halo_unique_id": ([vp, C.c_size_t], C.c_int),
        "mace_halo_create": ([vp, C.c_size_t, i32, i32, i32, C.POINTER(vp)], C.c_int),
        "mace_halo_plan": ([vp, i64, i64, i64, vp, vp, vp, vp], C.c_int),
        "mace_halo_destroy": ([vp], C.c_int),
        "mace_profile_enable": ([vp, i32], C.c_int),
        "mace_profile_read": ([vp, i32, C.c_char_p, C.POINTER(i32), C.POINTER(i32), C.POINTER(C.c_double),
                               C.POINTER(i32)], C.c_int),
        "mace_profile_timeline": ([vp, i32, C.c_char_p, C.POINTER(i32), C.POINTER(i32), C.POINTER(C.c_float),
                                   C.POINTER(C.c_float), C.POINTER(i32)], C.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    if path is None:
        _lib = lib
    return lib


def last_error(lib=None) -> str:
    lib = lib or load_library()
    buf = C.create_string_buffer(1024)
    lib.mace_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, lib=None) -> None:
    if rc != MACE_OK:
        raise NativeError(rc, last_error(lib))
