"""The allocation-free sign-mask entry point (b2p_sign_masks_noalloc) on the B200.

Callers that cannot allocate device memory (every device byte owned by another
allocator, or a fixed budget) use b2p_sign_masks_noalloc, whose scratch is a
fixed array inside the library. Its masks must equal, bit for bit, those of the
allocating entry point b2p_sign_masks on two calls in a row (the shared
scratch keeps the previous call's contents), and a ragged layout with 1-bit
tails must match the oracle. This file is collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from autoane_b200 import _lib
from autoane_b200.model import Config, Model
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def noalloc(sizes, seeds):
    sz = np.ascontiguousarray(sizes, np.int64)
    sd = np.ascontiguousarray(seeds, np.uint64)
    words = (int(sz.sum()) + 31) // 32
    out = torch.full((len(sd), words), -1, dtype=torch.int32, device="cuda")  # garbage the call must clear
    _lib.call("b2p_sign_masks_noalloc", sz.ctypes.data_as(C.POINTER(C.c_int64)), len(sz),
              sd.ctypes.data_as(C.POINTER(C.c_uint64)), len(sd), out.data_ptr(), None)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint32)


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


def test_noalloc_rejects_oversized_layout(b2p):
    with pytest.raises(_lib.B2PError, match="at most"):
        noalloc([4 * 524_288 + 4], [1])
