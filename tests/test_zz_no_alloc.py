"""The allocation-free AdamW entry point, called through its exported C symbol.

Callers that cannot allocate device memory (a runtime that owns a fixed arena, a loop
where a cudaMalloc would synchronize the device, a plain C host with no PyTorch
allocator) use ``tfb_adamw_multi_noalloc`` (declared in ``csrc/kernels/noalloc_adamw.h``):
its only scratch is a static table inside the library.  These tests call it through
ctypes and check every result against the regular ``adamw_multi`` entry point on
identical copies of the state: two calls in a row, then a call over fewer tensors than
the last one (the table keeps the earlier call's entries past its end), the cautious
weight-decay form, and a warmed-up call that must leave the device's free memory and
PyTorch's allocator untouched.  The file is named so pytest collects it last.
"""
import ctypes
import glob
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _lib():
    import trainium_frontier_b200._C  # noqa: F401  (loads torch's libraries first)
    paths = glob.glob(os.path.join(ROOT, "trainium_frontier_b200", "_C*.so"))
    assert paths, "sm_100a extension not built"
    lib = ctypes.CDLL(paths[0])
    f = lib.tfb_adamw_multi_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.POINTER(ctypes.c_void_p)] * 4 + [
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float),
        ctypes.c_int, ctypes.c_void_p, ctypes.c_double, ctypes.c_double, ctypes.c_float, ctypes.c_float,
        ctypes.c_int, ctypes.c_void_p]
    lib.tfb_adamw_noalloc_last_error.restype = ctypes.c_char_p
    lib.tfb_adamw_noalloc_max_tensors.restype = ctypes.c_int
    return lib


def _ptrs(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _call(lib, ps, gs, ms, vs, lr, b1, b2, eps, wd, bc1, bc2, n=None, cautious=0):
    n = len(ps) if n is None else n
    numels = (ctypes.c_longlong * len(ps))(*[t.numel() for t in ps])
    fb1 = (ctypes.c_float * len(ps))(*bc1)
    fb2 = (ctypes.c_float * len(ps))(*bc2)
    stream = torch.cuda.current_stream().cuda_stream
    return lib.tfb_adamw_multi_noalloc(_ptrs(ps), _ptrs(gs), _ptrs(ms), _ptrs(vs), numels, fb1, fb2, n,
                                       ctypes.c_void_p(lr.data_ptr()), b1, b2, eps, wd, cautious,
                                       ctypes.c_void_p(stream))


def test_noalloc_adamw_matches_regular_entry_point():
    from trainium_frontier_b200.ops.optim_kernels import adamw_multi
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib()
    torch.manual_seed(123)
    shapes = [(1280, 1280), (7,), (8192, 64), (3, 5, 11)]
    ps = [torch.randn(s, device=dev) for s in shapes]
    ms = [torch.randn(s, device=dev).abs() * 0.01 for s in shapes]
    vs = [torch.randn(s, device=dev).abs() * 0.01 for s in shapes]
    ps2, ms2, vs2 = [t.clone() for t in ps], [t.clone() for t in ms], [t.clone() for t in vs]
    lr = torch.tensor(3e-3, device=dev)
    b1, b2, eps, wd = 0.8, 0.95, 1e-10, 0.01
    for step in (1, 2):  # two calls in a row on the shared static table
        gs = [torch.randn(s, device=dev) for s in shapes]
        bc1 = [1 - b1 ** step] * len(ps)
        bc2 = [1 - b2 ** step] * len(ps)
        rc = _call(lib, ps, gs, ms, vs, lr, b1, b2, eps, wd, bc1, bc2)
        assert rc == 0, lib.tfb_adamw_noalloc_last_error()
        adamw_multi(ps2, gs, ms2, vs2, lr, b1, b2, eps, wd, bc1, bc2)
        torch.cuda.synchronize()
        for a, b in zip(ps + ms + vs, ps2 + ms2 + vs2):
            torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-7)


def test_noalloc_adamw_rejects_oversize_table():
    dev = torch.device("cuda", 0)
    lib = _lib()
    limit = lib.tfb_adamw_noalloc_max_tensors()
    t = torch.zeros(4, device=dev)
    lr = torch.tensor(1e-3, device=dev)
    ps = [t] * (limit + 1)
    rc = _call(lib, ps, ps, ps, ps, lr, 0.9, 0.95, 1e-8, 0.0, [1.0] * len(ps), [1.0] * len(ps))
    assert rc == 1
    assert b"exceeds" in lib.tfb_adamw_noalloc_last_error()
    assert torch.count_nonzero(t).item() == 0


def test_noalloc_adamw_shorter_call_cautious_and_no_allocation():
    from trainium_frontier_b200.ops.optim_kernels import adamw_multi
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib()
    torch.manual_seed(7)
    shapes = [(4096, 33), (5,), (1280, 512), (9, 9)]
    ps = [torch.randn(s, device=dev) for s in shapes]
    ms = [torch.randn(s, device=dev) * 0.01 for s in shapes]
    vs = [torch.randn(s, device=dev).abs() * 0.01 for s in shapes]
    ps2, ms2, vs2 = [t.clone() for t in ps], [t.clone() for t in ms], [t.clone() for t in vs]
    lr = torch.tensor(2e-3, device=dev)
    b1, b2, eps, wd = 0.9, 0.95, 1e-8, 0.1

    def both(idx, step, cautious):
        gs = [torch.randn(shapes[i], device=dev) for i in idx]
        bc1 = [1 - b1 ** step] * len(idx)
        bc2 = [1 - b2 ** step] * len(idx)
        sel = lambda ts: [ts[i] for i in idx]  # noqa: E731
        rc = _call(lib, sel(ps), gs, sel(ms), sel(vs), lr, b1, b2, eps, wd, bc1, bc2, cautious=cautious)
        assert rc == 0, lib.tfb_adamw_noalloc_last_error()
        adamw_multi(sel(ps2), gs, sel(ms2), sel(vs2), lr, b1, b2, eps, wd, bc1, bc2, bool(cautious))
        torch.cuda.synchronize()
        for a, b in zip(ps + ms + vs, ps2 + ms2 + vs2):
            torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-7)

    both([0, 1, 2, 3], 1, 0)   # all four tensors
    both([2, 0], 2, 0)         # then a shorter table, in another order
    both([1, 3, 0], 3, 1)      # cautious weight decay
    # A warmed-up call allocates nothing: neither through PyTorch's allocator nor on the device.
    gs = [torch.randn(s, device=dev) for s in shapes]
    torch.cuda.synchronize()
    alloc0 = torch.cuda.memory_allocated(dev)
    free0, _ = torch.cuda.mem_get_info(dev)
    rc = _call(lib, ps, gs, ms, vs, lr, b1, b2, eps, wd, [1 - b1 ** 4] * 4, [1 - b2 ** 4] * 4)
    torch.cuda.synchronize()
    assert rc == 0, lib.tfb_adamw_noalloc_last_error()
    assert torch.cuda.memory_allocated(dev) == alloc0
    assert torch.cuda.mem_get_info(dev)[0] == free0
