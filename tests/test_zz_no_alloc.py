"""The allocation-free sign-mask entry point (b2p_sign_masks_noalloc) on the B200.

Callers that cannot allocate device memory (every device byte owned by another
allocator, or a fixed budget) use b2p_sign_masks_noalloc, whose scratch is a
fixed array inside the library. Its masks must equal, bit for bit, those of the
allocating entry point b2p_sign_masks on two calls in a row (the shared
scratch keeps the previous call's contents), and a ragged layout with 1-bit
tails must match the oracle. Once the first call has set the array up, later
calls must not change the device's free memory. This file is collected last on
purpose.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from autoane_b200 import _lib
from autoane_b200.model import Config, Model
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def call_noalloc(sizes, seeds, out, stream=None):
    sz = np.ascontiguousarray(sizes, np.int64)
    sd = np.ascontiguousarray(seeds, np.uint64)
    _lib.call("b2p_sign_masks_noalloc", sz.ctypes.data_as(C.POINTER(C.c_int64)), len(sz),
              sd.ctypes.data_as(C.POINTER(C.c_uint64)), len(sd), C.c_void_p(out), stream)


def noalloc(sizes, seeds, stream=None):
    words = (int(np.sum(sizes)) + 31) // 32
    out = torch.full((len(seeds), words), -1, dtype=torch.int32, device="cuda")  # garbage the call must clear
    s = stream if stream is not None else torch.cuda.current_stream()
    s.wait_stream(torch.cuda.current_stream())
    call_noalloc(sizes, seeds, out.data_ptr(), C.c_void_p(s.cuda_stream) if stream is not None else None)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint32)


def test_noalloc_first_call_on_nonblocking_stream(b2p):
    """The first call of the process fills the jump table; a kernel it launches on a
    non-blocking stream (torch streams are) must already see the whole table."""
    sizes = O.lora_buffer_sizes(32, 960, 960, 320, 8)
    seeds = [5, 2**63 + 11]
    got = noalloc(sizes, seeds, stream=torch.cuda.Stream())
    for i, s in enumerate(seeds):
        assert np.array_equal(got[i], O.sign_mask(s, sizes)), f"seed {s}"


def test_noalloc_equals_allocating_path_on_consecutive_calls(b2p):
    model = Model(Config(max_groups=2))  # SmolLM2-360M LoRA layout (1,700,800 parameters)
    sizes = O.lora_buffer_sizes(32, 960, 960, 320, 8)
    for seeds in ([42, 1 * 1000003 + 42, 7], [2**64 - 1, 12345]):
        ref = model.sign_masks(seeds)
        got = noalloc(sizes, seeds)
        assert got.shape == ref.shape
        assert np.array_equal(got, ref), f"seeds {seeds}"
    model.close()


def test_noalloc_ragged_layout_matches_oracle(b2p):
    sizes = [7, 13, 8, 1, 3, 4, 5, 0, 2]
    for seeds in ([12345, 99], [3]):
        got = noalloc(sizes, seeds)
        for i, s in enumerate(seeds):
            assert np.array_equal(got[i], O.sign_mask(s, sizes)), f"seed {s}"


def test_noalloc_calls_leave_free_memory_unchanged(b2p):
    """After a warm-up call, repeated calls take no device memory (no cudaMalloc,
    no lazily created pool) — the property this entry point exists for."""
    sizes = O.lora_buffer_sizes(32, 960, 960, 320, 8)
    words = (int(np.sum(sizes)) + 31) // 32
    out = torch.empty((64, words), dtype=torch.int32, device="cuda")
    call_noalloc(sizes, [1], out.data_ptr())
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    launches0 = int(_lib.load().b2p_launch_count())
    for k in range(8):
        call_noalloc(sizes, list(range(k, k + 64)), out.data_ptr())
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert int(_lib.load().b2p_launch_count()) - launches0 >= 8


def test_noalloc_rejects_oversized_layout(b2p):
    with pytest.raises(_lib.B2PError, match="at most"):
        noalloc([4 * 524_288 + 4], [1])


def test_noalloc_rejects_host_output(b2p):
    host = np.zeros(4, np.uint32)
    with pytest.raises(_lib.B2PError, match="device memory"):
        call_noalloc([8], [1], host.ctypes.data)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_noalloc_rejects_other_device_output(b2p):
    """A buffer on another GPU is refused before any launch (it would be written over
    peer access, or fault without it)."""
    out = torch.zeros(4, dtype=torch.int32, device="cuda:1")
    with pytest.raises(_lib.B2PError, match="current"):
        call_noalloc([8], [1], out.data_ptr())
