"""C-ABI checks that need no GPU: the library loads, exports every symbol the header
declares, its argument structs match the Python mirror, and invalid arguments are
rejected with a status code and a message before any CUDA call."""
import ctypes
import os
import re

import pytest

from motif_ssm import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "motif_ssm.h")


def header_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^MSS_API [^(]*?\b(\w+)\(", src, flags=re.M)))


def test_header_declares_what_binding_binds():
    declared = header_functions()
    bound = sorted(name for name, _, _ in _lib.SYMBOLS)
    assert declared == bound


@pytest.mark.parametrize("name", header_functions())
def test_library_exports_symbol(name):
    assert hasattr(_lib.lib, name)


def test_struct_layouts_match_library():
    _lib.check_layout()
    sizes = (ctypes.c_int64 * 5)()
    _lib.lib.ss_abi_struct_sizes(sizes)
    assert list(sizes) == [ctypes.sizeof(s) for s in _lib.STRUCTS]


def test_constants():
    assert _lib.lib.ss_chunk_len() == 256
    assert _lib.lib.ss_max_dstate() >= 16
    assert b"sm_100a" in _lib.lib.ss_version()


def _fwd_args(**kw):
    a = _lib.SsFwdArgs()
    a.batch, a.dim, a.seqlen, a.dstate, a.n_groups = 2, 64, 256, 16, 1
    a.itype = _lib.MSS_BF16
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_fwd_rejects_null_struct():
    assert _lib.lib.ss_fwd(None, None) == _lib.MSS_ERR_INVALID
    assert b"null" in _lib.lib.ss_last_error()


@pytest.mark.parametrize("field,value,code", [
    ("itype", 7, _lib.MSS_ERR_INVALID),
    ("dstate", 0, _lib.MSS_ERR_INVALID),
    ("dstate", 300, _lib.MSS_ERR_UNSUPPORTED),
    ("n_groups", 3, _lib.MSS_ERR_INVALID),
    ("batch", -1, _lib.MSS_ERR_INVALID),
])
def test_fwd_rejects_bad_sizes(field, value, code):
    a = _fwd_args(**{field: value})
    assert _lib.lib.ss_fwd(ctypes.byref(a), None) == code
    assert _lib.lib.ss_last_error() != b""


def test_fwd_rejects_null_tensors():
    a = _fwd_args()
    assert _lib.lib.ss_fwd(ctypes.byref(a), None) == _lib.MSS_ERR_INVALID
    assert b"non-null" in _lib.lib.ss_last_error()


def test_fwd_empty_is_noop():
    a = _fwd_args(seqlen=0)
    assert _lib.lib.ss_fwd(ctypes.byref(a), None) == _lib.MSS_OK


def test_fwd_workspace_policy():
    """Large batch*dim runs in one pass (no workspace); small batch*dim with a long
    sequence is split into segments whose carries need a workspace."""
    nb = ctypes.c_int64(-1)
    a = _fwd_args(batch=32, dim=3072, seqlen=4096)
    assert _lib.lib.ss_fwd_workspace_size(ctypes.byref(a), ctypes.byref(nb)) == 0 and nb.value == 0
    a = _fwd_args(batch=1, dim=512, seqlen=32768)
    assert _lib.lib.ss_fwd_workspace_size(ctypes.byref(a), ctypes.byref(nb)) == 0 and nb.value > 0


def test_bwd_rejects_large_dstate_and_mismatched_grads():
    a = _lib.SsBwdArgs()
    a.batch, a.dim, a.seqlen, a.dstate, a.n_groups, a.itype = 1, 8, 64, 300, 1, _lib.MSS_F32
    assert _lib.lib.ss_bwd(ctypes.byref(a), None) == _lib.MSS_ERR_UNSUPPORTED
    a.dstate = 16
    a.D = 1234  # D given without dD
    assert _lib.lib.ss_bwd(ctypes.byref(a), None) == _lib.MSS_ERR_INVALID


def test_conv_rejects_width():
    a = _lib.Conv1dArgs()
    a.batch, a.dim, a.seqlen, a.width, a.itype, a.wtype = 1, 4, 8, 5, 0, 0
    assert _lib.lib.conv1d_fwd(ctypes.byref(a), None) == _lib.MSS_ERR_UNSUPPORTED


def test_state_update_rejects_groups():
    a = _lib.StateUpdateArgs()
    a.batch, a.dim, a.dstate, a.n_groups, a.itype, a.stype = 1, 6, 16, 4, 0, 0
    assert _lib.lib.ssm_state_update(ctypes.byref(a), None) == _lib.MSS_ERR_INVALID


def test_python_shim_raises_on_unbuilt_paths():
    import torch
    from motif_ssm import selective_scan_fn
    u = torch.zeros(1, 2, 4)
    A = -torch.ones(2, 4)
    B = torch.zeros(1, 4, 4)
    with pytest.raises(NotImplementedError):      # complex A
        selective_scan_fn(u, u, torch.complex(A, A), B, B)
    with pytest.raises(NotImplementedError):      # complex A on the P/Q path
        selective_scan_fn(u, u, torch.complex(A, A), B, B, P=torch.zeros(4, 2), Q=torch.zeros(2, 4))
    with pytest.raises(ValueError):               # P without Q
        selective_scan_fn(u, u, A, B, B, P=torch.zeros(4, 2))


def test_motif_regular_validates_before_launch():
    a = _lib.MotifRegularArgs()
    a.n_mat, a.cc = 1, 33
    assert _lib.lib.motif_regular(ctypes.byref(a), None) == _lib.MSS_ERR_UNSUPPORTED
    a.cc = 16
    assert _lib.lib.motif_regular(ctypes.byref(a), None) == _lib.MSS_ERR_INVALID  # null pointers
    a.n_mat = 0
    assert _lib.lib.motif_regular(ctypes.byref(a), None) == 0  # empty batch: no-op
    import torch
    from motif_ssm.motif_regular import motifRegular
    reg = motifRegular([0.25] * 13, device="cpu")
    assert reg.sum == 560 and reg.P.sum().item() == 16 * 15
    with pytest.raises(RuntimeError):  # no CPU path
        reg.cal(torch.zeros(16, 16), amplitude=1e5, bias=5e-5)
    with pytest.raises(ValueError):
        motifRegular([0.25] * 13, device="cpu", loss_weights=[1.0] * 12)
