"""Context behaviour at the C ABI on the GPU: each kq_ctx keeps its own device error word (a
second ctx on the same GPU neither clears nor sees the first one's error), and no entry point
leaves the caller on another GPU than the one it found."""
import ctypes

import pytest
import torch

import kernite_b200 as kb

pytestmark = pytest.mark.gpu


def _current_device() -> int:
    return torch.cuda.current_device()


def test_error_word_is_per_ctx():
    torch.cuda.set_device(0)
    a = kb.Kernels.load(0)
    try:
        # a counter nothing adds to: the bounded wait runs out (about 2 s) and records the error
        # in a's word, without faulting anything
        mem = torch.zeros(2, dtype=torch.int64, device="cuda")
        mem[1] = 1  # epoch 1: target = 0 * mul + add = 1, the counter stays 0
        a.wait_counter(mem.data_ptr(), mem.data_ptr() + 8, 0, 1)
        torch.cuda.synchronize()
        b = kb.Kernels.load(0)  # creating another ctx must not clear a's word
        try:
            b.device_error()  # b's own word is clear
        finally:
            b.close()
        with pytest.raises(kb.Error) as e:
            a.device_error()
        assert e.value.code == kb.KQ_E_DEVICE
        assert "another GPU's flag" in e.value.message
        a.device_error()  # read-and-clear: clear now
    finally:
        a.close()


def test_entry_points_give_back_the_callers_device():
    n = torch.cuda.device_count()
    other = 1 if n > 1 else 0
    torch.cuda.set_device(0)
    k = kb.Kernels.load(other)  # ctx creation makes its device current, as Cuda::on does
    try:
        torch.cuda.set_device(0)
        y = torch.zeros(16, device=f"cuda:{other}")
        x = torch.randn(256, device=f"cuda:{other}")
        W = torch.zeros(16 * 144, dtype=torch.uint8, device=f"cuda:{other}")
        k.fill(4, W, 0, 16, kb.stream_key(1, 4))
        assert _current_device() == 0
        k.matvec(4, y, W, x, 16, 256, 1)
        assert _current_device() == 0
        k.device_error()
        assert _current_device() == 0
        dev = ctypes.c_int(-1)
        L = kb.lib()
        L.kq_ctx_info(ctypes.c_void_p(k.handle), ctypes.byref(dev), None, None)
        assert dev.value == other
    finally:
        k.close()
    assert _current_device() == 0
