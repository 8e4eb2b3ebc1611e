"""GPU: ne_stream_read, the read-only floor the bench compares the decode
attention with, reads every chunk of its buffer exactly once."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nbytes", [16, 8192 * 3 + 48, 64 << 20])
def test_stream_read_touches_every_chunk(nbytes):
    import torch
    from neural_engine_b200 import runtime as rt
    lib = rt.load_library()
    g = torch.Generator().manual_seed(nbytes)
    host = torch.randint(-2**31, 2**31 - 1, (nbytes // 4,), dtype=torch.int32, generator=g)
    buf = host.cuda()
    sink = torch.zeros(2, dtype=torch.int32, device="cuda")
    assert lib.ne_stream_read(buf.data_ptr(), nbytes, sink.data_ptr(), None) == 0
    torch.cuda.synchronize()
    # chunks start at every multiple of 8 KB (per-warp ranges are whole chunks)
    want = np.bitwise_xor.reduce(host.numpy()[::2048].view(np.uint32))
    assert int(sink[1].item()) == 0
    assert np.uint32(sink[0].item() & 0xFFFFFFFF) == want


def test_stream_read_rejects_unaligned():
    import torch
    from neural_engine_b200 import runtime as rt
    lib = rt.load_library()
    buf = torch.zeros(64, dtype=torch.uint8, device="cuda")
    sink = torch.zeros(2, dtype=torch.int32, device="cuda")
    assert lib.ne_stream_read(buf.data_ptr(), 24, sink.data_ptr(), None) != 0
    assert lib.ne_stream_read(buf.data_ptr() + 8, 16, sink.data_ptr(), None) != 0
