"""ps_normalize_noalloc: the normalisation entry point for callers that cannot
allocate device memory when they call it (a framework whose pool owns all
device memory, a real-time loop that must stay out of the CUDA allocator, a
foreign runtime that holds device pointers but no allocator). Its scratch is a
static array inside the library instead of a caller workspace.

Checked through the C ABI against ps_normalize (the workspace entry point) on
two calls in a row -- bit for bit, since both use the same chunking when the
partial sums fit the scratch -- and against the CPU oracle with the
per-element FP16 tolerance the other kernel tests use. A batch whose partial
sums would not fit takes fewer, longer chunks: its bits may then differ from
ps_normalize in the last place, so that case is held to the oracle alone.
This file sorts last so a run that stops at the first failure has already run
every other test; it also passes when run alone in a fresh process.
"""

import pytest
import torch

from oracle import circuit as oc
from polar_switch import _native as nat
from tests._util import assert_fp16_close, seeded

pytestmark = pytest.mark.gpu

LIMIT = 32768  # PS_NORMALIZE_NOALLOC_MAX_PARTIALS in include/polar_switch_b200.h


def _call_noalloc(X, out, eps=1e-7):
    L, rows, cols = X.shape
    sL, sR, sC = X.stride()
    return nat.load().ps_normalize_noalloc(
        nat.ptr(X), nat.DTYPE_CODES[X.dtype], L, rows, cols, sL, sR, sC, float(eps),
        nat.ptr(out), out.shape[1], out.shape[2], nat.stream_ptr(X.device))


def _call_workspace(X, out, eps=1e-7):
    lib = nat.load()
    L, rows, cols = X.shape
    sL, sR, sC = X.stride()
    ws_bytes = lib.ps_normalize_workspace_bytes(L, rows, cols)
    ws = torch.empty(ws_bytes, device=X.device, dtype=torch.uint8)
    return lib.ps_normalize(nat.ptr(X), nat.DTYPE_CODES[X.dtype], L, rows, cols, sL, sR, sC,
                            float(eps), nat.ptr(out), out.shape[1], out.shape[2], nat.ptr(ws),
                            ws_bytes, nat.stream_ptr(X.device))


def _padded(X, device):
    L, rows, cols = X.shape
    rp, cp = -(-rows // 8) * 8, -(-cols // 8) * 8
    return torch.full((L, rp, cp), float("nan"), device=device, dtype=torch.float16)


def test_noalloc_normalize_matches_workspace_entry_point_and_oracle(cuda_device):
    cases = [seeded((6, 384, 520), 201, scale=2.0),            # first call: many partial sums
             seeded((2, 130, 66), 202, dtype=torch.bfloat16)]  # second call: fewer, padded output
    with torch.cuda.device(cuda_device):
        for i, X in enumerate(cases):
            Xd = X.to(cuda_device)
            L, rows, cols = Xd.shape
            got = _padded(Xd, cuda_device)
            ref = _padded(Xd, cuda_device)
            rc = _call_noalloc(Xd, got)
            assert rc == nat.PS_OK, nat.load().ps_last_error()
            assert _call_workspace(Xd, ref) == nat.PS_OK
            torch.cuda.synchronize()
            # the same chunking as ps_normalize: the same bits
            assert torch.equal(got, ref), f"noalloc call {i} differs from ps_normalize"
            assert_fp16_close(got[:, :rows, :cols], oc.normalize(X, 1e-7), max_ulps=1, max_mismatch=0.01,
                              what=f"noalloc call {i} vs oracle")
            assert torch.equal(got[:, rows:, :].float(), torch.zeros_like(got[:, rows:, :].float()))
            assert torch.equal(got[:, :, cols:].float(), torch.zeros_like(got[:, :, cols:].float()))
        assert nat.get_status() == 0


def test_noalloc_batch_beyond_the_canonical_chunking(cuda_device):
    """16400 matrices of 64 x 200 (two canonical chunks each, 32800 partial
    sums > the scratch): the entry point reduces each matrix over one longer
    chunk instead; the result is still the oracle's normalisation."""
    L, rows, cols = 16400, 64, 200
    assert L * 2 > LIMIT and L <= LIMIT
    X = seeded((L, rows, cols), 203, dtype=torch.float16, scale=3.0)
    with torch.cuda.device(cuda_device):
        Xd = X.to(cuda_device)
        got = _padded(Xd, cuda_device)
        for _ in range(2):  # two calls in a row share the scratch
            rc = _call_noalloc(Xd, got)
            assert rc == nat.PS_OK, nat.load().ps_last_error()
        torch.cuda.synchronize()
        assert nat.get_status() == 0
    assert_fp16_close(got.cpu(), oc.normalize(X, 1e-7), max_ulps=1, max_mismatch=0.01,
                      what="noalloc reduced chunking vs oracle")


def test_noalloc_rejects_batches_beyond_its_scratch(cuda_device):
    X = torch.zeros(8, device=cuda_device, dtype=torch.float32)
    out = torch.zeros(8, device=cuda_device, dtype=torch.float16)
    with torch.cuda.device(cuda_device):
        rc = nat.load().ps_normalize_noalloc(
            nat.ptr(X), nat.PS_F32, LIMIT + 1, 1, 1, 1, 1, 1, 1e-7, nat.ptr(out), 1, 1,
            nat.stream_ptr(cuda_device))
    assert rc == nat.PS_ERR_UNSUPPORTED
    assert b"exceed the built-in scratch" in nat.load().ps_last_error()
