"""The C-ABI library loads without a GPU and exports every symbol the header declares."""
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def declared():
    text = (ROOT / "include" / "enigma_cuda.h").read_text()
    return sorted(set(re.findall(r"^int32_t\s+(enigma_\w+)\s*\(", text, re.M)))


def test_library_exports_header():
    from enigma import _native
    lib = _native.lib()
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_prototypes_match_header():
    from enigma import _native
    assert sorted(_native.PROTOTYPES) == declared()


def test_status_without_gpu_is_an_error_not_a_crash():
    import ctypes
    from enigma import _native
    n = ctypes.c_int32(-1)
    rc = _native.lib().enigma_device_count(ctypes.byref(n))
    assert rc in (0, _native.ERR_EXEC, _native.ERR_DEVICE) and n.value >= 0
    rc = _native.lib().enigma_rmsnorm(7, None, None, None, 1, 1, ctypes.c_float(0.0), None)
    assert rc == _native.ERR_BADARG
    assert "dtype" in _native.last_error()
