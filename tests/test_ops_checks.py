"""The Python front end checks every buffer it hands to the library as a raw
pointer: exact element count, element size, contiguity and device, so that a
mis-shaped tensor is a ValueError on the host, never an out-of-bounds access
on the GPU.  These checks need no GPU."""
import pytest
import torch

from tqkv import ops


def test_need_accepts_exact_buffers():
    like = torch.zeros(4)
    ops._need(torch.zeros((2, 3), dtype=torch.int8), "t", 6, 1, like)
    ops._need(torch.zeros((3, 2), dtype=torch.float16), "t", 6, 2, like)
    ops._need(torch.zeros(12, dtype=torch.float16)[2:8], "t", 6, 2, like)   # offset view
    ops._need(torch.zeros((0, 5), dtype=torch.int8), "t", 0, 1, like)


@pytest.mark.parametrize("t,numel,esize", [
    (torch.zeros(5, dtype=torch.int8), 6, 1),             # too few elements
    (torch.zeros(7, dtype=torch.int8), 6, 1),             # too many
    (torch.zeros(6, dtype=torch.float16), 6, 1),          # wrong element size
    (torch.zeros((3, 4), dtype=torch.int8)[:, :2], 6, 1),  # not contiguous
])
def test_need_rejects(t, numel, esize):
    with pytest.raises(ValueError):
        ops._need(t, "t", numel, esize, torch.zeros(1))


def test_need_rejects_missing_buffer():
    with pytest.raises(ValueError):
        ops._need(None, "t", 1, 1, torch.zeros(1))


def test_scale_counts_follow_the_block_size():
    like = torch.zeros(1)
    rows, D = 10, 128
    for bs in (32, 64, 128):
        ops._check_scales(torch.zeros((rows, D // bs), dtype=torch.float16), "s", rows, D, bs,
                          like)
        with pytest.raises(ValueError):
            ops._check_scales(torch.zeros((rows, D // bs + 1), dtype=torch.float16), "s", rows, D,
                              bs, like)
    # block sizes the library rejects are left to its status code
    ops._check_scales(torch.zeros(1, dtype=torch.float16), "s", rows, D, 96, like)
    assert ops._nsub(128, 0) is None and ops._nsub(128, 96) is None and ops._nsub(64, 32) == 2


def test_wrappers_require_cuda_tensors():
    k = torch.zeros((1, 2, 8, 64), dtype=torch.int8)
    s = torch.zeros((1, 2, 8, 1), dtype=torch.float16)
    q = torch.zeros((1, 2, 64), dtype=torch.float16)
    with pytest.raises(ValueError):
        ops.decode_int8(q, k, s, k, s, 64)
