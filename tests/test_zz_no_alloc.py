"""The allocation-free BlockSparse encoder entry point.

Some callers of this library cannot allocate device memory (a host
application that owns every allocation, a memory pool that forbids
cudaMalloc), so `ngl_bs_encode_noalloc` keeps its scratch in a fixed device
array.  This test calls it through its exported C symbol and checks that two
calls in a row produce exactly the bytes of the regular encoder.  It lives in
its own file, collected last, and passes alone or after the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from mini_nangila_b200 import _ext

    lib = ctypes.CDLL(_ext.cuda().__file__)
    f = lib.ngl_bs_encode_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_void_p]
    lib.ngl_bs_encode_noalloc_max_n.restype = ctypes.c_int64
    lib.ngl_bs_encode_noalloc_error.restype = ctypes.c_char_p
    lib.ngl_bs_encode_noalloc_error.argtypes = [ctypes.c_int]
    return lib


def _codes(n, seed, sparsity):
    g = np.random.default_rng(seed)
    q = (g.standard_normal(n) * 300).astype(np.int16)
    q[g.random(n) < sparsity] = 0
    return torch.from_numpy(q).cuda()


def _noalloc_encode(lib, codes):
    n = codes.numel()
    nblk = (n + 31) // 32
    out = torch.zeros(4 + 68 * nblk, dtype=torch.uint8, device="cuda")
    total = torch.zeros(1, dtype=torch.int64, device="cuda")
    # Garbage in the status words: the entry point clears them itself, so a
    # caller need not.
    status = torch.full((4,), -7, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    ptr = codes.data_ptr() if n else 0
    rc = lib.ngl_bs_encode_noalloc(ptr, n, out.data_ptr(), total.data_ptr(), status.data_ptr(), stream)
    assert rc == 0, lib.ngl_bs_encode_noalloc_error(rc).decode()
    torch.cuda.synchronize()
    assert int(status[0]) == 0, status.tolist()
    return out[: int(total.item())].cpu().numpy().tobytes()


def test_noalloc_matches_regular_encoder_two_calls():
    from mini_nangila_b200 import _ext

    lib = _lib()
    # Two calls in a row: the second (smaller, different sparsity) must not
    # see the first call's tile status left in the shared scratch.
    for n, seed, sp in ((1_000_003, 1, 0.6), (70_001, 2, 0.95)):
        codes = _codes(n, seed, sp)
        got = _noalloc_encode(lib, codes)
        ref = _ext.cuda().pack_codes(codes, 0).cpu().numpy().tobytes()
        assert got == ref


def test_noalloc_edge_sizes():
    """Empty input (header only), one code past a whole 16384-code tile,
    and the largest accepted size, which uses the whole scratch array."""
    from mini_nangila_b200 import _ext

    lib = _lib()
    empty = _noalloc_encode(lib, torch.zeros(0, dtype=torch.int16, device="cuda"))
    assert empty == b"\x00\x00\x00\x00"  # [u32 n = 0], total 4 bytes
    for n, seed, sp in ((16385, 3, 0.5), (lib.ngl_bs_encode_noalloc_max_n(), 4, 0.9)):
        codes = _codes(n, seed, sp)
        got = _noalloc_encode(lib, codes)
        ref = _ext.cuda().pack_codes(codes, 0).cpu().numpy().tobytes()
        assert got == ref
        del codes


def test_noalloc_rejects_oversized_input():
    lib = _lib()
    mx = lib.ngl_bs_encode_noalloc_max_n()
    assert mx == 1 << 26
    codes = torch.zeros(1, dtype=torch.int16, device="cuda")
    rc = lib.ngl_bs_encode_noalloc(codes.data_ptr(), mx + 1, 0, 0, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == -2
    assert b"exceeds" in lib.ngl_bs_encode_noalloc_error(rc)
