"""Device-buffer helpers for the GPU tests: torch allocates and copies (plumbing); every kernel under test runs from
libwindlass_cuda through its C ABI."""
import ctypes as C

import numpy as np


def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "the gpu tests need a CUDA device"
    return torch


def dev(a):
    torch = torch_cuda()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def empty(n, dtype="float32"):
    torch = torch_cuda()
    return torch.empty(n, dtype=getattr(torch, dtype), device="cuda")


def ptr(t):
    return C.c_void_p(t.data_ptr())


def host(t):
    torch = torch_cuda()
    torch.cuda.synchronize()
    return t.cpu().numpy()


def rel_l2(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def random_blocks(O, t, blocks, seed):
    """RandomBlocks of tests/IQuantTests.cs: random payload bytes with a chosen fp16 scale in each block."""
    rng = O.Rng(seed)
    bs, bb = O.layout(t)
    raw = np.frombuffer(bytes(rng.byte() for _ in range(blocks * bb)), dtype=np.uint8).copy()
    dbits = [0x3A00, 0x3E00, 0x3800, 0xB400, 0x3C00]
    for k in range(blocks):
        if t == O.IQ1_M:
            for i in range(4):
                hi = raw[k * bb + 48 + 2 * i + 1]
                raw[k * bb + 48 + 2 * i + 1] = (hi & 0x0F) | (((dbits[k % 5] >> (4 * i)) & 15) << 4)
        else:
            raw[k * bb] = dbits[k % 5] & 0xFF
            raw[k * bb + 1] = dbits[k % 5] >> 8
    return raw


IQ_TYPES = ("iq4_nl", "iq4_xs", "iq3_xxs", "iq3_s", "iq2_xxs", "iq2_xs", "iq2_s", "iq1_s", "iq1_m")


def weights(O, tname, rows, cols, seed=3, rms=0.5):
    """Test weights of any decodable type: TinyModels.Matrix for float/legacy/K types, RandomBlocks for I-quants."""
    t = O.TYPE_OF[tname]
    if tname in IQ_TYPES:
        bs, _ = O.layout(t)
        return random_blocks(O, t, rows * cols // bs, seed)
    return O.matrix(O.Rng(seed), t, rows, cols, rms)
