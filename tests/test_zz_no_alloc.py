"""qcau_decode_attn_paged_noalloc against qcau_decode_attn_paged.

The no-alloc entry point runs the same kernels with the same split counts as
the workspace entry point, with the split-KV partials in the library's static
device scratch instead of a caller workspace, so its output must be the same
bytes.  Two calls in a row with different inputs (different lengths, so the
second call finds the first call's partials, in another layout, in the
scratch) check that nothing in the scratch has to start at zero.

This file is collected last so that it also runs after every other test has
used the library in the same process.
"""
from __future__ import annotations

import pytest
import torch

from qcau_b200 import _lib

PAGE, WIDTH, D_V = 64, 576, 512


def _case(seed, h, seqlens):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    b = len(seqlens)
    max_pages = max(1, (max(seqlens) + PAGE - 1) // PAGE)
    pages = b * max_pages + 3
    cache = torch.randn(pages, PAGE, WIDTH, device="cuda", generator=gen)
    cache = (cache * torch.rsqrt(cache.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    table = torch.randperm(pages, device="cuda", generator=gen)[:b * max_pages]
    table = table.view(b, max_pages).to(torch.int32).contiguous()
    q = torch.randn(b, h, WIDTH, device="cuda", generator=gen).to(torch.bfloat16)
    sink = torch.randn(h, device="cuda", generator=gen)
    sl = torch.tensor(seqlens, device="cuda", dtype=torch.int32)
    return dict(q=q, cache=cache, table=table, seqlens=sl, sink=sink, max_seqlen=max(seqlens),
                o=torch.empty(b, h, D_V, device="cuda", dtype=torch.bfloat16))


def _args(c):
    b, h, _ = c["q"].shape
    return (c["q"].data_ptr(), c["cache"].data_ptr(), c["table"].data_ptr(),
            c["seqlens"].data_ptr(), c["sink"].data_ptr(), c["o"].data_ptr(), b, h, WIDTH, D_V,
            WIDTH, PAGE, c["table"].size(1), c["cache"].size(0), c["max_seqlen"], 192 ** -0.5)


def _with_workspace(c):
    L = _lib.lib()
    b, h, _ = c["q"].shape
    need = L.qcau_decode_attn_workspace_size(b, h, D_V, c["max_seqlen"])
    ws = torch.empty(max(need, 1), device="cuda", dtype=torch.uint8)
    _lib.check(L.qcau_decode_attn_paged(*_args(c), ws.data_ptr(), need, _lib.stream_ptr()),
               "decode_attn_paged")
    torch.cuda.synchronize()
    return c["o"].clone()


def _noalloc(c):
    L = _lib.lib()
    _lib.check(L.qcau_decode_attn_paged_noalloc(*_args(c), _lib.stream_ptr()),
               "decode_attn_paged_noalloc")


# (128 heads: the tcgen05 two-CTA kernel over one 128-head group; 16 heads: the
# same kernel as a 16-head shard)
@pytest.mark.gpu
@pytest.mark.parametrize("h,first,second", [
    (128, [4096, 64, 777, 1], [0, 130, 2000]),
    (16, [1, 100, 1000, 3000], [513, 0, 64]),
])
def test_noalloc_matches_workspace_entry_point_twice(h, first, second):
    L = _lib.lib()
    c1, c2 = _case(11 + h, h, first), _case(23 + h, h, second)
    for c in (c1, c2):
        b = c["q"].size(0)
        assert L.qcau_decode_attn_workspace_size(b, h, D_V, c["max_seqlen"]) <= \
            _lib.DECODE_STATIC_SCRATCH_BYTES
    ref1, ref2 = _with_workspace(c1), _with_workspace(c2)
    c1["o"].fill_(0)
    c2["o"].fill_(0)
    torch.cuda.synchronize()

    # The first call on a device resolves the scratch's device address; the
    # array itself was placed when the library's module was loaded (the
    # workspace calls above already loaded it), so it is not counted here.
    _noalloc(c1)
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    _noalloc(c2)
    torch.cuda.synchronize()
    free_after = torch.cuda.mem_get_info()[0]

    assert torch.equal(c1["o"], ref1), "first no-alloc call differs from the workspace path"
    assert torch.equal(c2["o"], ref2), "second no-alloc call differs from the workspace path"
    assert free_after == free_before, "the no-alloc call changed the device's free memory"
    assert _lib.device_error() == 0


@pytest.mark.gpu
def test_noalloc_rejects_oversize_before_launch():
    """batch 128 x 128 heads at 32K context needs ~134 MB of partials, more
    than the static scratch holds: the call is refused before any launch.
    Every buffer is a real allocation of the size the call names (a one-page
    cache that the all-zero block table points at), so the only thing wrong
    with the call is the scratch size."""
    L = _lib.lib()
    b, h, ctx = 128, 128, 32768
    need = L.qcau_decode_attn_workspace_size(b, h, D_V, ctx)
    assert need > _lib.DECODE_STATIC_SCRATCH_BYTES
    q = torch.zeros(b, h, WIDTH, device="cuda", dtype=torch.bfloat16)
    o = torch.empty(b, h, D_V, device="cuda", dtype=torch.bfloat16)
    cache = torch.zeros(1, PAGE, WIDTH, device="cuda", dtype=torch.bfloat16)
    table = torch.zeros(b, ctx // PAGE, device="cuda", dtype=torch.int32)
    seqlens = torch.full((b,), ctx, device="cuda", dtype=torch.int32)
    o.fill_(1.0)
    torch.cuda.synchronize()
    rc = L.qcau_decode_attn_paged_noalloc(q.data_ptr(), cache.data_ptr(), table.data_ptr(),
                                          seqlens.data_ptr(), None, o.data_ptr(), b, h, WIDTH,
                                          D_V, WIDTH, PAGE, table.size(1), cache.size(0), ctx,
                                          0.07, _lib.stream_ptr())
    with pytest.raises(ValueError, match="static scratch"):
        _lib.check(rc, "decode_attn_paged_noalloc")
    assert str(need).encode() in L.qcau_last_error()
    torch.cuda.synchronize()
    assert bool((o == 1.0).all()), "the refused call wrote its output"
