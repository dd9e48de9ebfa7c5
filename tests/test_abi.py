"""The C ABI library loads and exports every entry point include/p2p_attn.h declares, and its
host-side validation fails with statuses (never an abort) -- all without a GPU."""
import ctypes as C
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "p2p_attn.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(p2p_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    import p2p_b200
    names = declared_functions()
    assert len(names) >= 20
    lib = C.CDLL(str(p2p_b200.LIB_PATH))
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(p2p_b200.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (p2p_\w+)", out))
    assert set(names) <= exported
    # the python bindings cover the whole header
    from p2p_b200._lib import PROTOTYPES
    assert set(names) == set(PROTOTYPES)


def test_abi_version_and_status_strings():
    from p2p_b200 import lib
    assert lib.p2p_abi_version() == 2
    for s in range(8):
        assert lib.p2p_status_string(s)
    assert lib.p2p_status_string(3) == b"kv cache full"


def test_null_and_invalid_arguments_return_status():
    from p2p_b200 import lib
    assert lib.p2p_ctx_create(0, None) == 1
    assert lib.p2p_ctx_destroy(None) == 1
    assert lib.p2p_kv_destroy(None) == 1
    assert lib.p2p_kv_capacity(None) == 0
    assert lib.p2p_kv_k(None, 0) is None
    assert lib.p2p_last_error(None) == b"no context"


def test_context_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from p2p_b200 import lib
    h = C.c_void_p()
    st = lib.p2p_ctx_create(0, C.byref(h))
    assert st == 4 and not h.value  # P2P_ERR_CUDA, no context


def test_communicator_host_side_without_gpu():
    """NCCL is loaded at run time; its unique id needs no GPU; bad arguments are statuses."""
    from p2p_b200 import lib
    from p2p_b200.comm import unique_id
    a, b = unique_id(), unique_id()
    assert len(a) == 128 and a != b
    h = C.c_void_p()
    assert lib.p2p_comm_create(None, 2, 0, a, 1000, C.byref(h)) == 1
    assert lib.p2p_comm_destroy(None) == 1
    assert lib.p2p_comm_wait(None, None) == 1
    assert lib.p2p_comm_barrier(None, None) == 1
    assert lib.p2p_attn_prefill_sharded(None, None, None, None, 0, None, None, None, None, 0,
                                        None, 0, 0, None, 0, None) == 1
    deps = subprocess.run(["ldd", str(ROOT / "p2p_b200" / "libp2pattn.so")],
                          capture_output=True, text=True).stdout
    assert "libnccl" not in deps  # dlopen'ed when a communicator is first needed


def test_product_library_does_not_link_the_oracle():
    import p2p_b200
    out = subprocess.run(["nm", "-D", str(p2p_b200.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    assert "p2p_or_" not in out
    deps = subprocess.run(["ldd", str(p2p_b200.LIB_PATH)], capture_output=True, text=True).stdout
    assert "oracle" not in deps
