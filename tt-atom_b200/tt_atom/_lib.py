"""ctypes binding of ``libatomb200.so`` (declarations in include/atom_b200.h).

The library must exist: there is no CPU or eager fallback. Every wrapper raises RuntimeError
with the library's own message when an entry point returns a non-zero status.
"""
from __future__ import annotations

import ctypes
import pathlib

import torch

_LIB_PATH = pathlib.Path(__file__).resolve().with_name("libatomb200.so")
_lib = None

ATOM_ERR_CAPACITY = 3
ATOM_ERR_UNSUPPORTED = 4

c_void_p, c_int, c_int64, c_float = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
c_double = ctypes.c_double


class CellGrid(ctypes.Structure):
    """atom_cell_grid of include/atom_b200.h."""
    _fields_ = [("inv_cell", c_double * 9), ("nb", c_int * 3), ("reach", c_int * 3),
                ("img_r", c_int * 3), ("atom_bin", c_void_p), ("atom_off", c_void_p),
                ("bin_cnt", c_void_p), ("bin_ptr", c_void_p), ("bin_atoms", c_void_p)]


class GemmGroups(ctypes.Structure):
    _fields_ = [("ngroups", c_int), ("a_col", c_int * 8), ("K", c_int * 8), ("c_col", c_int * 8),
                ("N", c_int * 8), ("ldb", c_int * 8), ("t_col", c_int * 8),
                ("B", c_void_p * 8), ("bias", c_void_p * 8), ("Bt", c_void_p * 8),
                ("Bt_lo", c_void_p * 8), ("Bh", c_void_p * 8), ("Bh_lo", c_void_p * 8),
                ("Bh_inv", c_void_p * 8)]


_SIGS = {
    "atom_last_error": (ctypes.c_char_p, ctypes.c_size_t),
    "atom_abi_version": (),
    "atom_launch_count": (ctypes.POINTER(c_int64),),
    "atom_fused_rotate": (c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_void_p,
                          c_void_p, c_void_p, c_void_p, c_void_p),
    "atom_fused_rotate_gc": (c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_void_p,
                             c_void_p, c_void_p, c_void_p),
    "atom_fused_gate": (c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_void_p,
                        c_void_p),
    "atom_fused_ln_bw": (c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float,
                         c_void_p, c_void_p),
    "atom_neighbor_list": (c_void_p, c_int64, c_void_p, c_int, c_void_p, c_int, c_float, c_int,
                           c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                           c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                           c_void_p),
    "atom_neighbor_refresh": (c_void_p, c_int64, c_void_p, c_int, c_float, c_int, c_int, c_int,
                              c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                              c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                              c_void_p),
    "atom_exclusive_scan": (c_void_p, c_int64, c_void_p, c_void_p, c_void_p),
    "atom_sender_csr": (c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p),
    "atom_sender_csr_noalloc": (c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p),
    "atom_edge_geometry": (c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p,
                           c_void_p, c_void_p, c_void_p, c_int, c_float, c_float, c_void_p,
                           c_void_p, c_void_p, c_void_p, c_void_p, c_void_p),
    "atom_edge_geometry_bwd": (c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                               c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_float, c_float,
                               c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p),
    "atom_forces_virial": (c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                           c_void_p, c_void_p, c_void_p, c_void_p),
    "atom_gemm": (c_void_p, c_int64, c_int64, ctypes.POINTER(GemmGroups), c_void_p, c_int64,
                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_int,
                  c_void_p),
    "atom_gemm_ex": (c_void_p, c_int64, c_int64, ctypes.POINTER(GemmGroups), c_void_p, c_int64,
                     c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int,
                     c_int, c_void_p, c_int64, c_void_p),
    "atom_gemm_gated": (c_void_p, c_int64, c_int64, ctypes.POINTER(GemmGroups), c_int, c_void_p,
                        c_int64, c_int, c_void_p, c_int64, c_void_p),
    "atom_device_error": (c_void_p, c_void_p),
    "atom_device_error_take": (c_void_p, c_void_p),
    "atom_wait_selftest": (c_int64, c_void_p),
    "atom_ring_wait_selftest": (c_int64, c_void_p),
    "atom_rotate_in": (c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_int64,
                       c_int, c_void_p, c_void_p, c_void_p),
    "atom_gate_fwd": (c_void_p, c_int64, c_int, c_void_p, c_void_p),
    "atom_gate_bwd": (c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p),
    "atom_rotate_back_reduce": (c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p,
                                c_void_p, c_void_p),
    "atom_rotate_back_bwd": (c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int,
                             c_void_p, c_void_p, c_void_p, c_void_p),
    "atom_rotate_in_bwd_edge": (c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p,
                                c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p,
                                c_void_p),
    "atom_rotate_in_bwd_node": (c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p,
                                c_int, c_void_p, c_void_p),
    "atom_edge_degree_fwd": (c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_int,
                             c_void_p, c_float, c_void_p, c_void_p),
    "atom_edge_degree_bwd": (c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64,
                             c_int, c_float, c_void_p, c_int64, c_void_p, c_void_p, c_void_p),
    "atom_ln_silu_fwd": (c_void_p, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p, c_float,
                         c_void_p, c_void_p),
    "atom_ln_silu_bwd": (c_void_p, c_void_p, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p,
                         c_float, c_void_p, c_void_p),
    "atom_rmsnorm_sh_fwd": (c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_float,
                            c_void_p, c_void_p),
    "atom_rmsnorm_sh_bwd": (c_void_p, c_void_p, c_int64, c_int, c_void_p, c_float, c_int,
                            c_void_p, c_void_p),
    "atom_node_project": (c_void_p, c_int64, c_int, c_int, c_void_p, c_int, c_int, c_int,
                          c_void_p, c_void_p),
    "atom_spectral_gate_fwd": (c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p),
    "atom_spectral_gate_bwd": (c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p,
                               c_void_p),
    "atom_silu_bwd": (c_void_p, c_void_p, c_int64, c_void_p, c_void_p),
    "atom_segment_sum": (c_void_p, c_int64, c_void_p, c_int, c_void_p, c_void_p),
    "atom_node_embed": (c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p,
                        c_void_p),
    "atom_orb_edge_features": (c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                               c_float, c_int, c_void_p, c_void_p, c_void_p, c_void_p),
    "atom_orb_edge_features_bwd": (c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                   c_float, c_int, c_void_p, c_void_p, c_void_p, c_void_p),
    "atom_rmsnorm_rows": (c_void_p, c_int64, c_int64, c_int, c_void_p, c_float, c_void_p,
                          c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p),
    "atom_rmsnorm_rows_bwd": (c_void_p, c_void_p, c_int64, c_int, c_void_p, c_float, c_void_p,
                              c_void_p),
    "atom_orb_attention": (c_void_p, c_int64, c_int, c_void_p, c_float, c_void_p, c_float,
                           c_void_p, c_void_p, c_void_p, c_void_p),
    "atom_csr_sum": (c_void_p, c_int64, c_void_p, c_int, c_void_p, c_void_p, c_int64, c_int,
                     c_void_p, c_int64, c_int, c_void_p),
    "atom_orb_messages_bwd": (c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                              c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p,
                              c_void_p, c_void_p, c_void_p),
    "atom_col_mean": (c_void_p, c_int64, c_int64, c_int, c_float, c_void_p, c_void_p),
    "atom_orb_zbl": (c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int, c_double,
                     c_void_p, c_void_p, c_void_p, c_void_p),
    "atom_row_broadcast": (c_void_p, c_int64, c_int, c_float, c_void_p, c_int64, c_int,
                           c_void_p),
    "atom_edge_species": (c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p),
}


def lib():
    """Load the kernel library (once). Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            raise RuntimeError(f"{_LIB_PATH.name} is not built; run `python -m tt_atom.build` "
                               "(this package has no CPU fallback)")
        L = ctypes.CDLL(str(_LIB_PATH))
        for name, args in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = list(args)
            f.restype = c_int
        _lib = L
    return _lib


def declared_symbols():
    return list(_SIGS)


def last_error():
    buf = ctypes.create_string_buffer(1024)
    lib().atom_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


class AtomError(RuntimeError):
    def __init__(self, name, code):
        super().__init__(f"{name} failed (status {code}): {last_error()}")
        self.code = code


def call(name, *args):
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise AtomError(name, rc)
    return rc


def check_device(stream=None):
    """Reads (and clears) the device-side error code of the tensor-core kernels and raises
    RuntimeError if a bounded wait expired since the last check: the results of every launch
    since then are incomplete and must not be returned. Synchronises the stream."""
    code = ctypes.c_int(0)
    call("atom_device_error", ctypes.byref(code), stream_ptr(stream))
    if code.value != 0:
        raise RuntimeError(
            f"a bounded device-side wait in the tensor-core GEMM expired (code {code.value}); "
            "the results of this evaluation are incomplete and were discarded")


def ptr(t):
    """Device pointer of a tensor (or None -> NULL)."""
    if t is None:
        return None
    return t.data_ptr()


def stream_ptr(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def host_i32(values):
    arr = (ctypes.c_int * len(values))(*[int(v) for v in values])
    return arr


def host_f32(values):
    return (ctypes.c_float * len(values))(*[float(v) for v in values])


def host_i64(values):
    return (ctypes.c_int64 * len(values))(*[int(v) for v in values])
