"""CPU checks of the boundary: the C-ABI library loads and exports every declared symbol,
and the Python bridge keeps the reference's names and signatures (no compute here)."""
import ctypes
import inspect
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "ltc_sm100.h")
LIB = os.path.join(REPO, "ltc-cuda_b200", "libltc_sm100.so")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ltc_[a-z_0-9]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        import importlib.util
        spec = importlib.util.spec_from_file_location("ltc_build", os.path.join(REPO, "ltc-cuda_b200", "build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    return ctypes.CDLL(LIB)


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("ltc_plan", "ltc_forward", "ltc_backward", "ltc_last_error", "ltc_version"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/ltc_sm100.h but not exported"


def test_version_and_error_without_gpu(lib):
    lib.ltc_version.restype = ctypes.c_int
    assert lib.ltc_version() >= 100
    lib.ltc_last_error.restype = ctypes.c_char_p
    assert isinstance(lib.ltc_last_error(), bytes)


def test_bridge_signatures_match_reference():
    import ltc_cuda
    # ltc_cuda.py:362-378 of the reference: 15 positional parameters
    params = list(inspect.signature(ltc_cuda.ltc_cuda_forward).parameters)
    assert params == ["x_seq", "state", "w_pos", "w_erev", "mu", "sigma", "sensory_mu", "sensory_sigma",
                      "sensory_erev", "sensory_w_pos", "cm_t", "gleak_pos", "vleak", "ode_unfolds", "epsilon"]
    fwd = list(inspect.signature(ltc_cuda.LTCCudaForward.forward).parameters)
    assert fwd[1:] == params + ["needs_grad"]
    assert hasattr(ltc_cuda, "_HAS_CUDA_KERNELS")
    for name in ("ltc_full_forward", "ltc_full_backward"):
        assert callable(getattr(ltc_cuda._cuda_module, name))
    # ctypes structures mirror the header's field lists
    src = open(HEADER).read()
    for struct, cls in (("LtcParams", ltc_cuda.LtcParams), ("LtcGrads", ltc_cuda.LtcGrads)):
        body = re.search(r"typedef struct \{([^{}]*)\} " + struct + ";", src, re.S).group(1)
        fields = re.findall(r"\*\s*([a-z_]+);", body)
        assert fields == [f for f, _ in cls._fields_], struct


def test_no_kernels_means_loud_error_without_cuda():
    import torch
    import ltc_cuda
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert ltc_cuda._HAS_CUDA_KERNELS is False
    with pytest.raises(RuntimeError):
        ltc_cuda.ltc_cuda_forward(*([torch.zeros(1)] * 13), 6, 1e-8)


def test_layer_state_dict_names_match_reference_module():
    import ltc_layer
    m = ltc_layer.TrueLiquidTimeConstant(10, 8)
    from golden_io import Case
    ref_keys = set(Case("verif_d10_h8").params)
    assert set(m.state_dict()) == ref_keys
