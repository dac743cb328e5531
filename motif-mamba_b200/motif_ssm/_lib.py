"""ctypes binding of the C ABI in ``include/motif_ssm.h`` (``libmotif_ssm.so``).

The structs below mirror the header field by field; ``check_layout()`` compares their
sizes with ``ss_abi_struct_sizes()`` exported by the library so a drift between the two
fails at load time instead of corrupting arguments.  There is no fallback: if the
library is missing the import raises.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("MOTIF_SSM_LIB", os.path.join(_HERE, "libmotif_ssm.so"))

MSS_OK, MSS_ERR_INVALID, MSS_ERR_UNSUPPORTED, MSS_ERR_ALIGNMENT, MSS_ERR_WORKSPACE, MSS_ERR_CUDA = range(6)
MSS_F32, MSS_F16, MSS_BF16 = 0, 1, 2

i64 = ctypes.c_int64
i32 = ctypes.c_int32
vp = ctypes.c_void_p


class SsFwdArgs(ctypes.Structure):
    _fields_ = [
        ("batch", i64), ("dim", i64), ("seqlen", i64), ("dstate", i64), ("n_groups", i64),
        ("itype", i32), ("delta_softplus", i32),
        ("u", vp), ("u_bs", i64), ("u_ds", i64),
        ("delta", vp), ("delta_bs", i64), ("delta_ds", i64),
        ("A", vp), ("A_ds", i64), ("A_ns", i64),
        ("B", vp), ("B_bs", i64), ("B_gs", i64), ("B_ns", i64),
        ("C", vp), ("C_bs", i64), ("C_gs", i64), ("C_ns", i64),
        ("D", vp), ("D_s", i64),
        ("delta_bias", vp), ("delta_bias_s", i64),
        ("z", vp), ("z_bs", i64), ("z_ds", i64),
        ("out", vp), ("out_bs", i64), ("out_ds", i64),
        ("out_z", vp), ("out_z_bs", i64), ("out_z_ds", i64),
        ("x", vp),
        ("workspace", vp), ("workspace_bytes", i64),
        ("P", vp), ("Q", vp),
        ("pq_rank", i64), ("pq_per_dim", i32), ("_pad_pq", i32),
        ("h0", vp),
    ]


class SsBwdArgs(ctypes.Structure):
    _fields_ = [
        ("batch", i64), ("dim", i64), ("seqlen", i64), ("dstate", i64), ("n_groups", i64),
        ("itype", i32), ("delta_softplus", i32), ("recompute_out_z", i32), ("_pad0", i32),
        ("u", vp), ("u_bs", i64), ("u_ds", i64),
        ("delta", vp), ("delta_bs", i64), ("delta_ds", i64),
        ("A", vp), ("A_ds", i64), ("A_ns", i64),
        ("B", vp), ("B_bs", i64), ("B_gs", i64), ("B_ns", i64),
        ("C", vp), ("C_bs", i64), ("C_gs", i64), ("C_ns", i64),
        ("D", vp), ("D_s", i64),
        ("delta_bias", vp), ("delta_bias_s", i64),
        ("z", vp), ("z_bs", i64), ("z_ds", i64),
        ("out", vp), ("out_bs", i64), ("out_ds", i64),
        ("x", vp),
        ("dout", vp), ("dout_bs", i64), ("dout_ds", i64),
        ("du", vp), ("du_bs", i64), ("du_ds", i64),
        ("ddelta", vp), ("ddelta_bs", i64), ("ddelta_ds", i64),
        ("dA", vp), ("dB", vp), ("dC", vp), ("dD", vp), ("ddelta_bias", vp),
        ("dz", vp), ("dz_bs", i64), ("dz_ds", i64),
        ("out_z", vp), ("out_z_bs", i64), ("out_z_ds", i64),
        ("workspace", vp), ("workspace_bytes", i64),
        ("P", vp), ("Q", vp),
        ("pq_rank", i64), ("pq_per_dim", i32), ("_pad_pq", i32),
        ("dP", vp), ("dQ", vp),
    ]


class Conv1dArgs(ctypes.Structure):
    _fields_ = [
        ("batch", i64), ("dim", i64), ("seqlen", i64), ("width", i64),
        ("itype", i32), ("wtype", i32), ("silu", i32), ("_pad0", i32),
        ("x", vp), ("x_bs", i64), ("x_ds", i64),
        ("weight", vp), ("w_ds", i64), ("w_ks", i64),
        ("bias", vp),
        ("out", vp), ("out_bs", i64), ("out_ds", i64),
        ("dout", vp), ("dout_bs", i64), ("dout_ds", i64),
        ("dx", vp), ("dx_bs", i64), ("dx_ds", i64),
        ("dweight", vp), ("dbias", vp),
    ]


class Conv1dUpdateArgs(ctypes.Structure):
    _fields_ = [
        ("batch", i64), ("dim", i64), ("width", i64), ("state_len", i64),
        ("itype", i32), ("wtype", i32), ("stype", i32), ("silu", i32),
        ("x", vp), ("x_bs", i64),
        ("conv_state", vp), ("cs_bs", i64), ("cs_ds", i64),
        ("weight", vp), ("w_ds", i64), ("w_ks", i64),
        ("bias", vp),
        ("out", vp), ("out_bs", i64),
    ]


class StateUpdateArgs(ctypes.Structure):
    _fields_ = [
        ("batch", i64), ("dim", i64), ("dstate", i64), ("n_groups", i64),
        ("itype", i32), ("stype", i32), ("dt_softplus", i32), ("_pad0", i32),
        ("state", vp), ("st_bs", i64), ("st_ds", i64), ("st_ns", i64),
        ("x", vp), ("x_bs", i64),
        ("dt", vp), ("dt_bs", i64),
        ("A", vp), ("A_ds", i64), ("A_ns", i64),
        ("B", vp), ("B_bs", i64), ("B_gs", i64),
        ("C", vp), ("C_bs", i64), ("C_gs", i64),
        ("D", vp),
        ("z", vp), ("z_bs", i64),
        ("dt_bias", vp),
        ("out", vp), ("out_bs", i64),
        ("state_batch_indices", vp), ("state_batch", i64),
    ]


class AddRmsNormArgs(ctypes.Structure):
    _fields_ = [
        ("rows", i64), ("dim", i64),
        ("itype", i32), ("rin_type", i32), ("rout_type", i32), ("wtype", i32),
        ("x", vp), ("x_rs", i64),
        ("residual_in", vp), ("rin_rs", i64),
        ("residual_out", vp), ("rout_rs", i64),
        ("weight", vp),
        ("out", vp), ("out_rs", i64),
        ("rstd", vp),
        ("eps", ctypes.c_float), ("_pad", i32),
    ]


class MotifRegularArgs(ctypes.Structure):
    _fields_ = [
        ("n_mat", i64), ("cc", i64),
        ("a", vp), ("a_ms", i64),
        ("target", vp), ("weight", vp),
        ("amplitude", ctypes.c_float), ("bias", ctypes.c_float),
        ("log_mse", i32), ("log_eps", ctypes.c_float),
        ("loss", vp), ("obs", vp), ("dloss", vp),
        ("da", vp), ("da_ms", i64),
    ]


class DtProjArgs(ctypes.Structure):
    _fields_ = [("dt_in", vp), ("dt_in_bs", i64), ("weight", vp), ("rank", i64)]


STRUCTS = (SsFwdArgs, SsBwdArgs, Conv1dArgs, Conv1dUpdateArgs, StateUpdateArgs)

# (name, argtypes, restype) of every symbol the header declares.
SYMBOLS = [
    ("ss_chunk_len", [], i32),
    ("ss_max_dstate", [], i32),
    ("ss_fwd_workspace_size", [ctypes.POINTER(SsFwdArgs), ctypes.POINTER(i64)], ctypes.c_int),
    ("ss_bwd_workspace_size", [ctypes.POINTER(SsBwdArgs), ctypes.POINTER(i64)], ctypes.c_int),
    ("ss_fwd", [ctypes.POINTER(SsFwdArgs), vp], ctypes.c_int),
    ("ss_bwd", [ctypes.POINTER(SsBwdArgs), vp], ctypes.c_int),
    ("ss_bwd_noalloc", [ctypes.POINTER(SsBwdArgs), vp], ctypes.c_int),
    ("conv1d_fwd", [ctypes.POINTER(Conv1dArgs), vp], ctypes.c_int),
    ("conv1d_bwd", [ctypes.POINTER(Conv1dArgs), vp], ctypes.c_int),
    ("conv1d_update", [ctypes.POINTER(Conv1dUpdateArgs), vp], ctypes.c_int),
    ("ssm_state_update", [ctypes.POINTER(StateUpdateArgs), vp], ctypes.c_int),
    ("ssm_state_update_dtproj", [ctypes.POINTER(StateUpdateArgs), ctypes.POINTER(DtProjArgs), vp], ctypes.c_int),
    ("add_rms_norm", [ctypes.POINTER(AddRmsNormArgs), vp], ctypes.c_int),
    ("add_rms_norm_args_size", [], i64),
    ("motif_regular", [ctypes.POINTER(MotifRegularArgs), vp], ctypes.c_int),
    ("motif_regular_args_size", [], i64),
    ("ss_last_error", [], ctypes.c_char_p),
    ("ss_version", [], ctypes.c_char_p),
    ("ss_abi_struct_sizes", [ctypes.POINTER(i64)], None),
]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"motif_ssm: native library not found at {LIB_PATH}; build it with "
            "`python motif-mamba_b200/build.py` (there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, argtypes, restype in SYMBOLS:
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    return lib


lib = _load()


def check_layout():
    sizes = (i64 * 5)()
    lib.ss_abi_struct_sizes(sizes)
    for s, st in zip(sizes, STRUCTS):
        if s != ctypes.sizeof(st):
            raise ImportError(f"motif_ssm: {st.__name__} is {ctypes.sizeof(st)} bytes in Python but {s} in the library")
    if lib.add_rms_norm_args_size() != ctypes.sizeof(AddRmsNormArgs):
        raise ImportError("motif_ssm: AddRmsNormArgs does not match add_rms_norm_args in the library")
    if lib.motif_regular_args_size() != ctypes.sizeof(MotifRegularArgs):
        raise ImportError("motif_ssm: MotifRegularArgs does not match motif_regular_args in the library")


check_layout()

_ERR_NAMES = {MSS_ERR_INVALID: "invalid argument", MSS_ERR_UNSUPPORTED: "unsupported",
              MSS_ERR_ALIGNMENT: "alignment", MSS_ERR_WORKSPACE: "workspace", MSS_ERR_CUDA: "CUDA error"}


class MotifSsmError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{msg} [{_ERR_NAMES.get(code, code)}]")
        self.code = code


def check(rc):
    if rc != MSS_OK:
        raise MotifSsmError(rc, lib.ss_last_error().decode())


CHUNK_LEN = lib.ss_chunk_len()
MAX_DSTATE = lib.ss_max_dstate()
VERSION = lib.ss_version().decode()
