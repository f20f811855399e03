"""GPU: ownership-tracked device buffers (mcb_device_*), the mirror of the
reference's DeviceBufferHandle / matcore_device_* (device_buffer.h:11-53):
round trips through the synchronous and stream-ordered copies, zeroing, and
stale-handle detection after free, also when the allocator hands the same
address out again."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _alloc(lib, abi, nbytes, device=0):
    h = abi.Buffer()
    assert lib.mcb_device_alloc(device, nbytes, ctypes.byref(h)) == 0
    assert lib.mcb_device_is_valid(h) == 1 and h.size_bytes == nbytes
    return h


def test_round_trip_sync_and_async(mcb):
    import torch
    from matcoredsl_b200 import _abi
    lib = mcb.load()
    n = 1 << 20
    h = _alloc(lib, _abi, n)
    src = np.random.default_rng(1).integers(0, 256, n, dtype=np.uint8)
    dst = np.zeros(n, np.uint8)
    assert lib.mcb_device_upload(h, src.ctypes.data, n) == 0
    assert lib.mcb_device_download(dst.ctypes.data, h, n) == 0
    assert np.array_equal(src, dst)
    # Stream-ordered copies from / to pinned memory on a torch stream.
    pin_src = torch.from_numpy(src[::-1].copy()).pin_memory()
    pin_dst = torch.zeros(n, dtype=torch.uint8).pin_memory()
    s = torch.cuda.Stream()
    assert lib.mcb_device_upload_async(h, pin_src.data_ptr(), n, s.cuda_stream) == 0
    assert lib.mcb_device_download_async(pin_dst.data_ptr(), h, n, s.cuda_stream) == 0
    s.synchronize()
    assert torch.equal(pin_src, pin_dst)
    # Sizes beyond the buffer are refused.
    assert lib.mcb_device_upload_async(h, pin_src.data_ptr(), n + 1, s.cuda_stream) != 0
    assert lib.mcb_device_zero(h) == 0
    assert lib.mcb_device_download(dst.ctypes.data, h, n) == 0
    assert not dst.any()
    assert lib.mcb_device_free(h) == 0


def test_freed_handle_is_stale_even_if_address_is_reused(mcb):
    from matcoredsl_b200 import _abi
    lib = mcb.load()
    stale = _abi.STATUS_CODE["STALE_HANDLE"]
    h1 = _alloc(lib, _abi, 4096)
    assert lib.mcb_device_free(h1) == 0
    assert lib.mcb_device_is_valid(h1) == 0
    buf = np.zeros(4096, np.uint8)
    assert lib.mcb_device_upload(h1, buf.ctypes.data, 4096) == stale
    assert lib.mcb_device_free(h1) == stale  # double free
    h2 = _alloc(lib, _abi, 4096)
    assert h2.alloc_id != h1.alloc_id
    # Whether or not the allocator returned the same address, only h2 is live.
    assert lib.mcb_device_is_valid(h1) == 0 and lib.mcb_device_is_valid(h2) == 1
    assert lib.mcb_device_free(h2) == 0
