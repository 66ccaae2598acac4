"""helm_copy_pages: scattered host pages gathered into consecutive device slots (one gather
kernel when the source is pinned and device-addressable), runs of consecutive ids merged into
single copies, and the cudaMemcpyAsync path for pageable or device sources -- every path bytewise
equal to torch indexing."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _pages(n, shape, pin):
    g = torch.Generator().manual_seed(n)
    t = torch.randn((n,) + shape, generator=g).to(torch.bfloat16)
    return t.pin_memory() if pin else t


@pytest.mark.parametrize("pin", [True, False])
def test_scattered_host_pages(pin):
    from helm_b200 import ops
    src = _pages(300, (2, 4, 64, 128), pin)
    page_bytes = src[0].numel() * 2
    ids = torch.randperm(300, generator=torch.Generator().manual_seed(1))[:180].tolist()
    dst = torch.zeros((200,) + src.shape[1:], dtype=src.dtype, device=DEV)
    n = ops.copy_pages(dst, 7, src, ids, page_bytes)
    torch.cuda.synchronize()
    assert torch.equal(dst[7:187].cpu(), src[ids])
    assert torch.equal(dst[:7].cpu(), torch.zeros_like(dst[:7].cpu()))
    assert torch.equal(dst[187:].cpu(), torch.zeros_like(dst[187:].cpu()))
    if pin:
        assert n == 1          # one gather launch
    else:
        assert n >= 16         # one copy per run


def test_runs_and_device_source():
    from helm_b200 import ops
    src = _pages(64, (2, 2, 64, 128), True)
    page_bytes = src[0].numel() * 2
    ids = list(range(10, 20)) + list(range(40, 45))          # two runs: copied with cudaMemcpyAsync
    dst = torch.zeros((40,) + src.shape[1:], dtype=src.dtype, device=DEV)
    assert ops.copy_pages(dst, 0, src, ids, page_bytes) == 2
    dsrc = src.to(DEV)
    ids2 = torch.randperm(64, generator=torch.Generator().manual_seed(2))[:20].tolist()
    assert ops.copy_pages(dst, 15, dsrc, ids2, page_bytes) >= 16   # device source: copies
    torch.cuda.synchronize()
    assert torch.equal(dst[:15].cpu(), src[ids])
    assert torch.equal(dst[15:35].cpu(), src[ids2])


@pytest.mark.parametrize("direction", ["d2h", "h2d", "d2d"])
def test_move_pages_scatter_gather(direction):
    """helm_move_pages: (source slot, destination slot) pairs in any order, one kernel for many runs,
    bytewise equal to torch indexing; destination slots not named stay untouched."""
    from helm_b200 import ops
    host = _pages(96, (2, 2, 64, 128), True)
    page_bytes = host[0].numel() * 2
    g = torch.Generator().manual_seed(5)
    src_ids = torch.randperm(96, generator=g)[:70].tolist()
    dst_ids = torch.randperm(80, generator=g)[:70].tolist()
    if direction == "d2h":
        src = host.to(DEV)
        dst = torch.zeros((80,) + host.shape[1:], dtype=host.dtype).pin_memory()
    elif direction == "h2d":
        src = host
        dst = torch.zeros((80,) + host.shape[1:], dtype=host.dtype, device=DEV)
    else:
        src = host.to(DEV)
        dst = torch.zeros((80,) + host.shape[1:], dtype=host.dtype, device=DEV)
    n = ops.move_pages(dst, dst_ids, src, src_ids, page_bytes)
    torch.cuda.synchronize()
    assert n == 1
    want = torch.zeros((80,) + host.shape[1:], dtype=host.dtype)
    want[dst_ids] = host[src_ids]
    assert torch.equal(dst.cpu(), want)


def test_move_pages_runs_use_copies():
    from helm_b200 import ops
    host = _pages(32, (2, 2, 64, 128), True)
    page_bytes = host[0].numel() * 2
    src = host.to(DEV)
    dst = torch.zeros((40,) + host.shape[1:], dtype=host.dtype).pin_memory()
    assert ops.move_pages(dst, list(range(5, 15)) + [30, 31], src, list(range(0, 10)) + [20, 21], page_bytes) == 2
    torch.cuda.synchronize()
    assert torch.equal(dst[5:15], host[0:10]) and torch.equal(dst[30:32], host[20:22])


def test_move_pages_rejects_out_of_range_ids():
    from helm_b200 import ops
    from helm_b200 import _native as N
    src = torch.zeros((8, 2, 2, 64, 128), dtype=torch.bfloat16, device=DEV)
    dst = torch.zeros((4, 2, 2, 64, 128), dtype=torch.bfloat16).pin_memory()
    with pytest.raises(N.HelmError):
        ops.move_pages(dst, [0, 4], src, [1, 2], src[0].numel() * 2)
    with pytest.raises(ValueError):
        ops.copy_pages(src, 7, dst, [0, 1], src[0].numel() * 2)
