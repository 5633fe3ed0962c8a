"""Host -> device staging (spmm_b200._device.to_device): arrays larger than a
staging buffer go through the two reused pinned buffers; the copy is exact,
ordered on the current stream, and converts the dtype first."""

import numpy as np
import pytest
import torch

from spmm_b200 import _device

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('n,dtype,to', [
    (1000, np.int32, None),                              # one pinned copy
    (_device.STAGE_BYTES // 8 * 5 + 3, np.int64, None),  # five and a bit buffers
    (_device.STAGE_BYTES // 4 * 3 + 1, np.int64, np.int32),
    (_device.STAGE_BYTES // 4 + 7, np.float32, None),
])
def test_staged_copy_is_exact(cuda, n, dtype, to):
    rng = np.random.default_rng(n)
    a = rng.integers(-2**30, 2**30, n).astype(dtype)
    want = a.astype(to) if to is not None else a
    got = _device.to_device(a, cuda, to)
    assert got.shape == (n,)
    np.testing.assert_array_equal(got.cpu().numpy(), want)


def test_back_to_back_copies_reuse_the_buffers(cuda):
    """Consecutive staged copies (and one on a side stream) do not overwrite
    each other's data in flight."""
    n = _device.STAGE_BYTES // 4 * 3
    arrays = [np.full(n, k, dtype=np.int32) for k in range(4)]
    side = torch.cuda.Stream(cuda)
    outs = [_device.to_device(arrays[0], cuda), _device.to_device(arrays[1], cuda)]
    with torch.cuda.stream(side):
        outs.append(_device.to_device(arrays[2], cuda))
    outs.append(_device.to_device(arrays[3], cuda))
    torch.cuda.synchronize()
    for k, o in enumerate(outs):
        assert bool((o == k).all())
