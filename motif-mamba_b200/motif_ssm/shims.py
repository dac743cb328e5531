"""Register this library under the module names the reference imports, so the
reference's own Python (``mamba_ssm``) runs on the sm_100a kernels unchanged:

* ``selective_scan_cuda``                          (``selective_scan_interface.py:21``)
* ``causal_conv1d`` and ``causal_conv1d.cpp_functions`` (``selective_scan_interface.py:10-17``,
  ``mamba_simplemotif.py:15-18``)
* ``mamba_ssm.ops.triton.selective_state_update`` (``mamba_simplemotif.py:21``) and
  ``mamba_ssm.ops.triton.layer_norm`` (``selective_scan_interface.py:19``) -- only the leaf
  modules are registered; their parent packages must already be importable.

Call ``install()`` before importing the reference's modules.
"""
import sys
import types

from . import causal_conv1d as _cc
from . import layer_norm as _ln
from . import selective_scan_cuda as _ssc
from . import selective_state_update as _ssu


def install():
    sys.modules["selective_scan_cuda"] = _ssc
    sys.modules["causal_conv1d"] = _cc
    cpp = types.ModuleType("causal_conv1d.cpp_functions")
    cpp.causal_conv1d_fwd_function = _cc.causal_conv1d_fwd_function
    cpp.causal_conv1d_bwd_function = _cc.causal_conv1d_bwd_function
    cpp.causal_conv1d_update_function = _cc.causal_conv1d_update_function
    sys.modules["causal_conv1d.cpp_functions"] = cpp
    sys.modules["mamba_ssm.ops.triton.selective_state_update"] = _ssu
    sys.modules["mamba_ssm.ops.triton.layer_norm"] = _ln
    return True
