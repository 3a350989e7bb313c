"""ca_decode_noalloc, the decode entry point for callers that cannot allocate
device memory (an engine that reserves all GPU memory up front, a plugin
interface that hands over only input and output buffers): it must give the
same output as ca_decode, which takes a caller-allocated workspace, call after
call, while allocating nothing itself.

Called through the C ABI directly (ctypes), twice in a row, against ca_decode
on the same inputs, within the tolerance the decode tests use (bf16 max-abs
2e-2, fp32 1e-4 relative; the two share one kernel, so they normally agree
exactly), and against the C restatement of the reference's kernel with the
same tolerance. After the first call (which looks up the scratch array's
address) the device's free memory does not move across further calls. This
file is collected last on purpose, and passes alone in a fresh process as well
as after the other tests.
"""

import ctypes

import pytest
import torch

from helpers import north_star_ok
from oracle import cpu as ORACLE

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(dtype, B, H, E, page, seed, maxlen=1500):
    """Caches filled through reshape_and_cache, lengths long enough that
    sequences split into pieces merged through the scratch's tickets."""
    import cpu_attention as C
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, maxlen, (B,), generator=g, dtype=torch.int32)
    W = -(-(maxlen + 1) // page)
    nblocks = B * W
    bt = torch.randperm(nblocks, generator=g).to(torch.int32).view(B, W)
    kc = torch.full((nblocks, H, page, E), float("nan"), dtype=dtype, device=DEV)
    vc = kc.clone()
    for i in range(B):
        n = int(lens[i])
        pos = torch.arange(n)
        slots = (bt[i, pos // page].long() * page + pos % page).to(DEV)
        C.reshape_and_cache(torch.randn(n, H, E, generator=g).to(dtype).to(DEV),
                            torch.randn(n, H, E, generator=g).to(dtype).to(DEV), kc, vc, slots)
    q = torch.randn(B, H, E, generator=g).to(dtype).to(DEV)
    kn = torch.randn(B, H, E, generator=g).to(dtype).to(DEV)
    vn = torch.randn(B, H, E, generator=g).to(dtype).to(DEV)
    return q, kc, vc, bt.to(DEV), lens.to(DEV), kn, vn


def _args(q, kc, vc, bt, lens, kn, vn, out):
    B, H, E = q.shape
    return (q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), kc.shape[0], kn.data_ptr(), vn.data_ptr(),
            kn.stride(0), None, lens.data_ptr(), bt.data_ptr(), bt.shape[1], out.data_ptr(), B, H, E, kc.shape[2],
            1 if q.dtype == torch.bfloat16 else 0, float("nan"))


@pytest.mark.parametrize("dtype,B,H,E,page", [(torch.bfloat16, 8, 16, 128, 16), (torch.float32, 6, 4, 64, 32)])
def test_noalloc_matches_decode_twice(dtype, B, H, E, page):
    from cpu_attention import _kernel as K
    lib = K.library()
    q, kc, vc, bt, lens, kn, vn = _case(dtype, B, H, E, page, seed=B * E)
    stream = torch.cuda.current_stream().cuda_stream
    # the existing entry point, with its own workspace
    need = lib.ca_decode_workspace_bytes(B, H, E, page, 1 if dtype == torch.bfloat16 else 0, q.device.index)
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    ref = torch.empty_like(q)
    assert lib.ca_decode(*_args(q, kc, vc, bt, lens, kn, vn, ref), ws.data_ptr(), ws.numel(), stream) == K.OK
    torch.cuda.synchronize()
    # the C restatement of the reference kernel on host copies (it appends the
    # new token at lens[i] too)
    cpu = torch.empty(q.shape, dtype=dtype)
    ORACLE.decode(q.cpu(), kc.cpu(), vc.cpu(), lens.cpu(), bt.cpu(), cpu, k_new=kn.cpu(), v_new=vn.cpu())
    # the allocation-free one, two calls in a row (the second reuses what the
    # first left in the shared scratch); outputs made before the calls, so
    # that nothing in the loop allocates
    outs = [torch.empty_like(q) for _ in range(3)]
    torch.cuda.synchronize()
    free = []
    for out in outs:
        assert lib.ca_decode_noalloc(*_args(q, kc, vc, bt, lens, kn, vn, out), stream) == K.OK
        torch.cuda.synchronize()
        free.append(torch.cuda.mem_get_info()[0])
        err, tol = north_star_ok(out, ref, dtype)
        assert err <= tol, err
        err, tol = north_star_ok(out, cpu, dtype)
        assert err <= tol, err
    assert free[1] == free[0] and free[2] == free[0], free


def test_noalloc_rejects_beyond_its_scratch():
    from cpu_attention import _kernel as K
    lib = K.library()
    p = ctypes.c_void_p(256)
    # batch * heads = 65537 > 65536: declined before any device work
    rc = lib.ca_decode_noalloc(p, 128 * 64, p, p, 8, None, None, 0, None, p, p, 1, p, 65537, 1, 64, 16, 1,
                               float("nan"), None)
    assert rc == K.ESCRATCH
