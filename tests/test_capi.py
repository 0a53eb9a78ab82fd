"""CPU tests of the C ABI: libtm_b200.so builds for sm_100a, loads, exports every entry point include/*.h declares,
and rejects malformed calls before touching a device (no compute without a GPU)."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names |= set(re.findall(r"^\s*(?:const\s+)?[\w\*\s]+?\b(tm_\w+)\s*\(", src, flags=re.M))
    return names


def test_header_declares_entry_points():
    d = declared()
    assert {"tm_launch", "tm_register", "tm_kernel_info", "tm_kernel_id"} <= d


def test_library_exports_every_declared_symbol(tmlib):
    L = tmlib.lib()
    for name in declared():
        assert hasattr(L, name), name
    assert set(tmlib.EXPORTS) <= declared()
    assert L.tm_abi_version() == 1


def test_builtin_kernels(tmlib):
    names = tmlib.kernel_names()
    for n in ("q1_fwd", "q1_grad", "rw_fwd", "rw_grad"):
        assert n in names
    from tallymap_b200 import backend as B
    for p in B.PROGRAMS.values():
        kid, nbuf = tmlib.kernel_id(p.kernel)
        if p.buffers:                                       # launched by its own driver (backend.tree_grad)
            assert nbuf == p.buffers, p.name
            continue
        layout, n_zero = p.result_layout(10)
        assert nbuf == p.n_args + len(layout), p.name       # the Python layout matches the kernel's


def test_replay_state_sizes_match_the_kernels(tmlib):
    """the host sizes each replay scratch by the program's replay_state_bytes: it must be the kernel's stored-state
    size, or the scratch would be too small for the states the kernel writes"""
    from tallymap_b200 import backend as B
    checked = 0
    for p in B.PROGRAMS.values():
        kid, _ = tmlib.kernel_id(p.kernel)
        n = ctypes.c_int32()
        tmlib.check(tmlib.lib().tm_kernel_state_bytes(kid, ctypes.byref(n)))
        if p.replay_state_bytes or n.value:
            assert n.value == p.replay_state_bytes, p.name
            checked += 1
    assert checked >= 6


def test_unknown_kernel_rejected(tmlib):
    with pytest.raises(tmlib.TallymapError, match="no built-in kernel"):
        tmlib.kernel_id("no_such_program")


def test_launch_rejects_bad_arguments(tmlib):
    kid, nbuf = tmlib.kernel_id("rw_fwd")
    L = tmlib.lib()
    bufs = (ctypes.c_void_p * nbuf)(*([1] * nbuf))
    rb = (ctypes.c_size_t * nbuf)(*([4] * nbuf))
    st = ctypes.c_int32()
    # wrong buffer count
    assert L.tm_launch(kid, None, bufs, 2, 2, rb, 0, 0, 10, ctypes.byref(st)) == tmlib.TM_EINVAL
    assert b"takes" in L.tm_last_error()
    # negative item count
    assert L.tm_launch(kid, None, bufs, 4, nbuf - 4, rb, 0, 0, -1, ctypes.byref(st)) == tmlib.TM_EINVAL
    # n_zero beyond the results
    assert L.tm_launch(kid, None, bufs, 4, nbuf - 4, rb, nbuf, 0, 10, ctypes.byref(st)) == tmlib.TM_EINVAL
    # unknown id
    assert L.tm_launch(12345, None, bufs, 4, nbuf - 4, rb, 0, 0, 10, ctypes.byref(st)) == tmlib.TM_EINVAL


def test_register_validates(tmlib):
    L = tmlib.lib()
    img = b"\x7fELF" + b"\0" * 60
    assert L.tm_register(99, img, len(img), b"x", 0, 0, 128) == tmlib.TM_EINVAL
    assert L.tm_register(99, img, len(img), b"x", 8, 0, 100) == tmlib.TM_EINVAL
    assert L.tm_register(99, None, 0, b"x", 8, 0, 128) == tmlib.TM_EINVAL


def test_check_status(tmlib):
    L = tmlib.lib()
    ok = (ctypes.c_uint32 * 8)()
    assert L.tm_check_status(ok) == tmlib.TM_OK
    bad = (ctypes.c_uint32 * 8)(0, 0, 0, 1, 0, 0, 0, 0)
    assert L.tm_check_status(bad) == tmlib.TM_EDEVICE
    assert b"timed out" in L.tm_last_error()


def test_product_path_has_no_cpu_fallback():
    """the package never imports the oracle, and refuses a non-CUDA target"""
    import tallymap_b200
    from tallymap_b200 import backend as B
    pkg = os.path.dirname(tallymap_b200.__file__)
    for f in glob.glob(os.path.join(pkg, "**", "*.py"), recursive=True):
        src = open(f).read()
        assert not re.search(r"^\s*(from\s+oracle|import\s+oracle)", src, flags=re.M), f
    with pytest.raises(NotImplementedError):
        B.run(B.RW_FWD, [], [], target="cpu")


def test_shower_claim_order_is_a_permutation():
    """the shower's claim order: every root once, largest primary energy first (host logic; no launch)"""
    import numpy as np
    import torch
    import tallymap_b200 as tm
    from tallymap_b200 import backend as B
    E = np.random.default_rng(5).exponential(size=1000).astype(np.float32)
    o = B.energy_order(E).numpy()
    assert o.dtype == np.int32 and np.array_equal(np.sort(o), np.arange(1000))
    assert np.all(np.diff(E[o]) <= 0)
    fo = tm.FAMILIES["shower"].claim_order([torch.from_numpy(E)])
    assert np.array_equal(fo.numpy(), o)
    assert all(tm.FAMILIES[n].claim_order is None for n in tm.FAMILIES if n != "shower")
