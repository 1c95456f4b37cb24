"""CPU checks of the C ABI: the library loads, exports exactly what
include/bee_b200.h declares, and validates arguments on the host (these calls
return before any CUDA API is touched, so they need no GPU)."""
import ctypes
import re
from pathlib import Path

import pytest

from bee_b200 import _capi

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "bee_b200.h"


def header_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"BEE_B200_API\s+[\w\s\*]+?\b(bee_b200_\w+)\s*\(", text)))


def test_header_declares_functions():
    names = header_functions()
    assert len(names) >= 20
    assert "bee_b200_ew_binary" in names and "bee_b200_reduce_global" in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_capi.LIB_PATH))
    missing = [n for n in header_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_binding_matches_header():
    assert sorted(_capi.SIGNATURES) == header_functions()


def test_version_and_status_strings():
    lib = _capi.lib()
    assert lib.bee_b200_version() >= 100
    assert lib.bee_b200_status_string(0) is not None


def _rc(name, *args):
    lib = _capi.lib()
    return getattr(lib, name)(*args), _capi.last_error()


def test_empty_inputs_are_noops_or_errors_like_the_reference():
    # size-0 elementwise is a successful no-op (Bee/CUDA/Api.cpp:213-214) ...
    assert _rc("bee_b200_ew_binary", 0, 4, None, None, None, 0, None)[0] == 0
    assert _rc("bee_b200_ew_cast", 4, None, 8, None, 0, None)[0] == 0
    # ... while an empty global / axis reduce is an error (Api.cpp:237-238, 245-246)
    rc, msg = _rc("bee_b200_reduce_global", 0, 2, None, None, 0, None)
    assert rc == 1 and "empty" in msg
    rc, msg = _rc("bee_b200_reduce_axis", 0, 4, None, None, 0, 4, 1, None)
    assert rc == 1 and "empty" in msg


@pytest.mark.parametrize("call", [
    ("bee_b200_ew_binary", 0, 4, None, None, None, 16, None),          # null pointers
    ("bee_b200_ew_binary", 0, 99, 16, 16, 16, 16, None),               # unknown dtype
    ("bee_b200_ew_binary", 9, 4, 16, 16, 16, 16, None),                # unknown op
    ("bee_b200_ew_unary", 2, 2, 16, 16, 16, None),                     # sqrt on int32
    ("bee_b200_ew_cast", 4, 16, 99, 16, 16, None),                     # unknown target dtype
    ("bee_b200_scale_fp", 2, 16, 2.0, 16, None),                       # scale on int32
    ("bee_b200_reduce_global", 0, 1, 16, 16, 16, None),                # sum on U8
    ("bee_b200_reduce_global", 7, 4, 16, 16, 16, None),                # unknown reduce op
    ("bee_b200_softmax_rows", 2, 16, 16, 4, 4, None),                  # softmax on int32
    ("bee_b200_softmax_rows", 4, 16, 16, 4, 0, None),                  # zero columns
    ("bee_b200_rms_norm_rows", 4, 16, 16, 16, 4, 4, -1.0, None),       # negative eps
    ("bee_b200_rope", 4, 16, 16, 8, 4, 2, 7, 10000.0, 0, None),        # odd head_dim
    ("bee_b200_rope", 4, 16, 16, 6, 4, 2, 8, 10000.0, 0, None),        # rows not a multiple of seq
    ("bee_b200_rope", 4, 16, 16, 8, 4, 2, 512, 10000.0, 0, None),      # head_dim too large
    ("bee_b200_rms_norm_rope", 4, 16, 16, 16, 8, 4, 2, 8, 1e-6, 0.0, 0, None),  # theta <= 0
    ("bee_b200_allocate", None, 16, 256, None),                        # null out pointer
    ("bee_b200_allocate", ctypes.pointer(ctypes.c_void_p()), 16, 512, None),  # alignment > 256
])
def test_host_side_validation(call):
    rc, msg = _rc(*call)
    assert rc == 1, (call[0], rc)
    assert msg, "a failed call must leave a message"


def test_success_clears_message():
    _rc("bee_b200_ew_binary", 0, 99, 16, 16, 16, 16, None)
    assert _capi.last_error()
    assert _rc("bee_b200_ew_binary", 0, 4, None, None, None, 0, None)[0] == 0
    assert _capi.last_error() == ""


def test_binding_raises_with_message():
    with pytest.raises(_capi.BeeError) as e:
        _capi.call("bee_b200_reduce_global", 0, 2, None, None, 0, None)
    assert e.value.status == 1 and "empty" in str(e.value)


def test_splitk_receive_buffer_size():
    lib = _capi.lib()
    # 8192 x 8192 -> 1024 tiles of 256 x 256; world 3 owns ceil(1024 / 3) = 342 per rank, 3 slots each
    assert lib.bee_b200_splitk_recv_bytes(8192, 8192, 3) == 3 * 342 * 65536 * 4
    assert lib.bee_b200_splitk_recv_bytes(1, 8, 1) == 65536 * 4
    assert lib.bee_b200_splitk_recv_bytes(520, 776, 2) == 2 * 6 * 65536 * 4  # 3 x 4 tiles
    assert lib.bee_b200_splitk_recv_bytes(8, 8, 0) == 0


def test_splitk_argument_checks_on_host():
    peers = (ctypes.c_void_p * 9)(*([16] * 9))
    rc, msg = _rc("bee_b200_gemm_splitk_scatter", 16, 64, 16, 64, 64, 64, peers, 9, 0, None)
    assert rc == 1 and "world" in msg
    rc, msg = _rc("bee_b200_gemm_splitk_scatter", 16, 64, 16, 64, 64, 64, peers, 2, 2, None)
    assert rc == 1 and "out of range" in msg
    rc, msg = _rc("bee_b200_gemm_splitk_scatter", 16, 64, 16, 64, 60, 64, peers, 2, 0, None)
    assert rc == 1 and "multiples of 8" in msg
    rc, msg = _rc("bee_b200_gemm_splitk_scatter", 16, 64, 16, 64, 0, 64, peers, 2, 0, None)
    assert rc == 1
    rc, msg = _rc("bee_b200_gemm_splitk_scatter", None, 64, 16, 64, 64, 64, peers, 2, 0, None)
    assert rc == 1 and "null" in msg
    rc, msg = _rc("bee_b200_gemm_splitk_reduce", 16, peers, 64, 60, 2, 0, None)
    assert rc == 1 and "multiple of 8" in msg
    assert _rc("bee_b200_gemm_splitk_reduce", 16, peers, 0, 64, 2, 0, None)[0] == 0  # empty C: no-op
    rc, msg = _rc("bee_b200_ipc_alloc", None, 16)
    assert rc == 1 and "null" in msg
