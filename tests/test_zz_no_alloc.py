"""Decode attention through the entry point that allocates nothing.

``hc_flash_decode_noalloc`` exists for callers that cannot allocate device
memory -- for example a host program whose device memory is all owned by
another allocator, or a language binding that has no device allocator to
call -- and so cannot hand ``hc_flash_decode`` its workspace.  It keeps the
split-K partials in a fixed array inside the library instead.

These tests call both entry points through the C ABI (ctypes, raw pointers)
on the same paged cache, on two calls in a row, so that a call which starts
from the previous call's leftovers in the shared array is covered too.  Both
entry points launch the same kernels with the same grid on the same inputs,
so their outputs must be identical bit for bit (stricter than the 2e-2
max-abs the decode-attention tests allow against the fp32 oracle).  The file sorts last so that a run stopping at the
first failure has already run every other test; it also passes on its own in
a fresh process.
"""
import ctypes

import pytest
import torch

from heterocache_b200 import _lib

pytestmark = pytest.mark.gpu

BF16 = 1


def _paged(lengths, kv=8, h=32, d=128, seed=0, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    nb = sum((l + 255) // 256 for l in lengths) + 2
    mb = max((l + 255) // 256 for l in lengths) + 1
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    bt = torch.full((len(lengths), mb), -1, dtype=torch.int32)
    ptr = 0
    for r, l in enumerate(lengths):
        n = (l + 255) // 256
        bt[r, :n] = perm[ptr:ptr + n]
        ptr += n
    kp = torch.randn(nb, 256, 1, d, generator=g).to(torch.bfloat16).to(device)
    vp = torch.randn(nb, 256, 1, d, generator=g).to(torch.bfloat16).to(device)
    bsz = len(lengths) // kv
    q = torch.randn(bsz, h, 1, d, generator=g).to(torch.bfloat16).to(device)
    return q, kp, vp, bt.to(device), torch.tensor(lengths, dtype=torch.int32, device=device)


def _call(lib, name, q, kp, vp, bt, hl, out, err, ws=None):
    bsz, h, _, d = q.shape
    kv = bt.shape[0] // bsz
    stream = torch.cuda.current_stream().cuda_stream
    common = (BF16, bsz, kv, h // kv, d, q.data_ptr(), q.stride(0), q.stride(1), kp.data_ptr(), vp.data_ptr(),
              kp.shape[0], bt.data_ptr(), bt.shape[1], hl.data_ptr(), ctypes.c_float(0.0), out.data_ptr())
    if name == "hc_flash_decode":
        return lib.hc_flash_decode(*common, 0, ws.data_ptr(), ws.numel(), err.data_ptr(), stream)
    return lib.hc_flash_decode_noalloc(*common, err.data_ptr(), stream)


def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    lib = _lib.lib()
    lens = [131, 4099, 0, 256, 17, 30000, 513, 2048]
    q, kp, vp, bt, hl = _paged(lens, seed=3)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ws = torch.zeros(lib.hc_flash_decode_workspace_size(1, 8, 4, 128), dtype=torch.uint8, device=cuda_device)
    for call in range(2):
        if call == 1:  # a second, different query on the same cache
            q = torch.randn_like(q.float()).to(torch.bfloat16)
        ref = torch.empty(1, 32, 128, dtype=torch.bfloat16, device=cuda_device)
        out = torch.full_like(ref, float("nan"))
        assert _call(lib, "hc_flash_decode", q, kp, vp, bt, hl, ref, err, ws) == 0
        assert _call(lib, "hc_flash_decode_noalloc", q, kp, vp, bt, hl, out, err) == 0
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert not torch.isnan(out.float()).any()
        diff = (out.float() - ref.float()).abs().max().item()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), (call, diff)


def test_noalloc_rejects_requests_beyond_its_scratch(cuda_device):
    """Too many rows for the fixed array: refused before anything is launched."""
    lib = _lib.lib()
    bsz, kv, g = 128, 8, 8
    h = kv * g
    q = torch.zeros(bsz, h, 1, 128, dtype=torch.bfloat16, device=cuda_device)
    kp = torch.zeros(1, 256, 1, 128, dtype=torch.bfloat16, device=cuda_device)
    bt = torch.zeros(bsz * kv, 1, dtype=torch.int32, device=cuda_device)
    hl = torch.zeros(bsz * kv, dtype=torch.int32, device=cuda_device)
    out = torch.full((bsz, h, 128), 7.0, dtype=torch.bfloat16, device=cuda_device)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    rc = _call(lib, "hc_flash_decode_noalloc", q, kp, kp, bt, hl, out, err)
    torch.cuda.synchronize()
    assert rc == 6  # HC_ERR_WORKSPACE
    assert b"fixed scratch" in lib.hc_last_cuda_error()
    assert out.float().eq(7.0).all()
