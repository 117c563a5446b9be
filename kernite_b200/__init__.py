"""kernite_b200 -- a B200-native Q4_K / Q5_K / Q6_K matvec behind kernite-cuda's call surface.

The product is ``libkq.so`` (hand-written CUDA for sm_100a behind the C ABI in
``include/kq.h``). This module is the host-side mirror of fxeqxmulfx/kernite's interface for the
path, bound with ctypes:

* :class:`Cuda` -- a GPU, as ``kernite_cuda::Cuda::on(i)`` (crates/cuda/src/lib.rs:570-617).
* :class:`Kernels` -- the loaded kernels, as a macro-generated ``Kernels::load(&cuda)``
  (crates/macros/src/gpu.rs:74-98), with one launcher per kernel, as the macro's
  ``unsafe fn <kernel>(&self, grid, params...) -> Result<(), Error>``
  (crates/macros/src/gpu.rs:276-328). The grid is the library's choice, so launchers take no grid.
* :class:`Error` -- ``kernite_cuda::Error{call, message, log}`` (crates/cuda/src/lib.rs:280-324).

Pointers are device addresses (``int``) or CUDA tensors (their ``data_ptr()``), the caller's
buffers; nothing here allocates for a launch. There is no CPU fallback: without ``libkq.so``
every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
from typing import Any

HERE = os.path.dirname(os.path.abspath(__file__))
# The in-tree build of the library (kernite_b200/build.py writes it).
LIB_PATH = os.path.join(HERE, "libkq.so")

KQ_OK = 0
KQ_E_INVALID = 1001
KQ_E_UNSUPPORTED = 1002
KQ_E_DEVICE = 1003
KQ_E_COMM = 1004

TYPE_Q4_K = 12
TYPE_Q5_K = 13
TYPE_Q6_K = 14
TYPE_Q8_0 = 8   # batch-1 matvec on the CUDA cores
TYPE_Q2_K = 10  # batch-1 matvec on the CUDA cores
TYPE_Q3_K = 11  # batch-1 matvec on the CUDA cores
PROLOGUE_NONE = 0
PROLOGUE_RMSNORM = 1
EPILOGUE_NONE = 0
EPILOGUE_PAIR_PRODUCT = 1
EPILOGUE_SILU_PRODUCT = 2
FLAG_WEIGHTS_STATIC = 1
FLAG_NO_PDL = 2
FLAG_TENSOR_CORES = 4
FLAG_CUDA_CORES = 8
FLAG_WARP_MMA = 16

Q4K_BYTES = 144
Q6K_BYTES = 210
Q5K_BYTES = 176
Q2K_BYTES = 84
Q3K_BYTES = 110
Q8_0_UNIT_BYTES = 272  # eight 34-byte Q8_0 blocks = 256 weights
QK = 256

# Every symbol include/kq.h declares (tests check the library exports each).
EXPORTS = (
    "kq_ctx_create", "kq_ctx_destroy", "kq_last_error", "kq_ctx_info", "kq_device_error",
    "kq_matvec_q4k", "kq_matvec_q6k", "kq_matvec", "kq_matvec_host", "kq_dequant_q4k", "kq_dequant_q6k",
    "kq_fill_q4k", "kq_fill_q6k", "kq_dequant_q5k", "kq_fill_q5k", "kq_dequant_q2k", "kq_dequant_q3k",
    "kq_dequant_q8_0", "kq_stream_key", "kq_matvec_q4k_noalloc",
    "kq_matvec_push", "kq_wait_counter", "kq_matvec_chain", "kq_epoch_advance", "kq_peer_alloc", "kq_peer_open", "kq_peer_close", "kq_peer_free",
    "kq_gguf_open", "kq_gguf_close", "kq_gguf_tensor_count", "kq_gguf_tensor_at", "kq_gguf_find",
    "kq_gguf_meta_int", "kq_gguf_meta_str", "kq_module_image", "kq_matvec_plan",
    "kq_rope_append", "kq_attention_decode", "kq_attention_workspace", "kq_tagged_unpack",
)


class Error(RuntimeError):
    """What went wrong in a call: ``call`` (the C function), ``message``, and ``code``."""

    def __init__(self, call: str, message: str, code: int = -1, log: str = ""):
        self.call = call
        self.message = message
        self.code = code
        self.log = log
        super().__init__(f"{call}: {message}" + (f"\n{log}" if log else ""))


class KqMatvecDesc(ctypes.Structure):
    _fields_ = [
        ("type", ctypes.c_uint32), ("rows", ctypes.c_uint32), ("k", ctypes.c_uint32),
        ("batch", ctypes.c_uint32), ("y", ctypes.c_uint64), ("w", ctypes.c_uint64),
        ("x", ctypes.c_uint64), ("ldx", ctypes.c_uint64), ("ldy", ctypes.c_uint64),
        ("prologue", ctypes.c_uint32), ("epilogue", ctypes.c_uint32), ("eps", ctypes.c_float),
        ("pair_scale", ctypes.c_float), ("flags", ctypes.c_uint32), ("reserved", ctypes.c_uint32),
    ]


class KqGgufTensor(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char_p), ("type", ctypes.c_uint32), ("n_dims", ctypes.c_uint32),
        ("dims", ctypes.c_uint64 * 4), ("offset", ctypes.c_uint64), ("nbytes", ctypes.c_uint64),
        ("data", ctypes.c_void_p),
    ]


class KqPushDesc(ctypes.Structure):
    _fields_ = [
        ("npush", ctypes.c_uint32), ("push_rows", ctypes.c_uint32),
        ("y", ctypes.c_uint64 * 8), ("counter", ctypes.c_uint64 * 8),
        ("wait_counter", ctypes.c_uint64), ("epoch", ctypes.c_uint64),
        ("wait_mul", ctypes.c_uint64), ("wait_add", ctypes.c_uint64),
        ("flags", ctypes.c_uint32), ("reserved", ctypes.c_uint32),
        ("push_mul", ctypes.c_uint64), ("push_add", ctypes.c_uint64),
        ("ksplit", ctypes.c_uint32), ("x_slots", ctypes.c_uint32),
    ]


PUSH_TAGGED = 1
PUSH_TAGGED_X = 2


class KqLaunch(ctypes.Structure):
    """``kq_launch`` (include/kq.h): one planned launch of a function of the module image."""
    _fields_ = [
        ("kernel", ctypes.c_char * 256), ("grid", ctypes.c_uint32 * 3), ("block", ctypes.c_uint32 * 3),
        ("shared_bytes", ctypes.c_uint32), ("param_bytes", ctypes.c_uint32),
        ("params", ctypes.c_uint8 * 512),
    ]


class KqChainJob(ctypes.Structure):
    """``kq_chain_job`` (include/kq.h): one matvec of a chain launch."""
    _fields_ = [
        ("mv", KqMatvecDesc), ("wait_counter", ctypes.c_uint64), ("wait_target", ctypes.c_uint64),
        ("npush", ctypes.c_uint32), ("push_rows", ctypes.c_uint32),
        ("push_y", ctypes.c_uint64 * 8), ("counter", ctypes.c_uint64 * 8),
    ]


CHAIN_MAX_JOBS = 8

IPC_HANDLE_BYTES = 64

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded ``libkq.so``; raises :class:`Error` if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise Error("dlopen", f"{LIB_PATH} is missing: build it with `python -m kernite_b200.build`")
    L = ctypes.CDLL(LIB_PATH)
    vp = ctypes.c_void_p
    u32, u64, i32 = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int
    L.kq_ctx_create.argtypes = [i32, ctypes.POINTER(vp)]
    L.kq_ctx_destroy.argtypes = [vp]
    L.kq_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    L.kq_last_error.restype = ctypes.c_size_t
    L.kq_ctx_info.argtypes = [vp, ctypes.POINTER(i32), ctypes.POINTER(i32), ctypes.POINTER(i32)]
    L.kq_device_error.argtypes = [vp]
    for name in ("kq_matvec_q4k", "kq_matvec_q6k"):
        getattr(L, name).argtypes = [vp, u64, u64, u64, u32, u32, u32, vp]
    L.kq_matvec.argtypes = [vp, ctypes.POINTER(KqMatvecDesc), vp]
    L.kq_matvec_host.argtypes = [vp, ctypes.POINTER(KqMatvecDesc), vp, vp, vp]
    for name in ("kq_dequant_q4k", "kq_dequant_q5k", "kq_dequant_q6k", "kq_dequant_q2k",
                 "kq_dequant_q3k", "kq_dequant_q8_0"):
        getattr(L, name).argtypes = [vp, u64, u64, u64, vp]
    for name in ("kq_fill_q4k", "kq_fill_q5k", "kq_fill_q6k"):
        getattr(L, name).argtypes = [vp, u64, u64, u64, u64, vp]
    L.kq_stream_key.argtypes = [u64, u64]
    L.kq_stream_key.restype = u64
    L.kq_matvec_q4k_noalloc.argtypes = [u64, u64, u64, u32, u32, u32, vp]
    L.kq_matvec_push.argtypes = [vp, ctypes.POINTER(KqMatvecDesc), ctypes.POINTER(KqPushDesc), vp]
    L.kq_wait_counter.argtypes = [vp, u64, u64, u64, u64, vp]
    L.kq_tagged_unpack.argtypes = [vp, u64, u64, u64, u64, u64, u64, vp]
    L.kq_matvec_chain.argtypes = [vp, ctypes.POINTER(KqChainJob), u32, u64, vp]
    L.kq_module_image.argtypes = [ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_size_t)]
    L.kq_rope_append.argtypes = [vp, u64, u64, u64, u64, u32, u32, u32, u32, ctypes.c_double, vp]
    L.kq_attention_decode.argtypes = [vp, u64, u64, u64, u64, u32, u32, u32, u32, u64, u64, vp]
    L.kq_attention_workspace.argtypes = [vp, u32, u32, u32, u32]
    L.kq_attention_workspace.restype = u64
    L.kq_matvec_plan.argtypes = [vp, ctypes.POINTER(KqMatvecDesc), ctypes.POINTER(KqLaunch)]
    L.kq_epoch_advance.argtypes = [vp, u64, vp]
    L.kq_peer_alloc.argtypes = [vp, u64, ctypes.POINTER(u64), ctypes.c_char_p]
    L.kq_peer_open.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(u64)]
    L.kq_peer_close.argtypes = [vp, u64]
    L.kq_peer_free.argtypes = [vp, u64]
    L.kq_gguf_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(vp)]
    L.kq_gguf_close.argtypes = [vp]
    L.kq_gguf_tensor_count.argtypes = [vp]
    L.kq_gguf_tensor_count.restype = u64
    L.kq_gguf_tensor_at.argtypes = [vp, u64, ctypes.POINTER(KqGgufTensor)]
    L.kq_gguf_find.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(KqGgufTensor)]
    L.kq_gguf_meta_int.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)]
    L.kq_gguf_meta_str.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p)]
    for name in EXPORTS:
        fn = getattr(L, name)
        if name not in ("kq_last_error", "kq_stream_key", "kq_gguf_tensor_count", "kq_attention_workspace"):
            fn.restype = i32
    _lib = L
    return L


def last_error() -> str:
    L = lib()
    n = L.kq_last_error(None, 0)
    buf = ctypes.create_string_buffer(n + 1)
    L.kq_last_error(buf, n + 1)
    return buf.value.decode(errors="replace")


def _check(rc: int, call: str) -> None:
    if rc != 0:
        msg = last_error()
        head, _, rest = msg.partition(": ")
        raise Error(head or call, rest or msg, rc)


def _addr(p: Any) -> int:
    if p is None:
        return 0
    if isinstance(p, int):
        return p
    if hasattr(p, "data_ptr"):
        if hasattr(p, "is_cuda") and not p.is_cuda:
            raise Error("kernite_b200", "a tensor given as a device pointer is on the CPU")
        return int(p.data_ptr())
    raise TypeError(f"not a device pointer: {type(p)!r}")


def _host_addr(p: Any) -> int:
    """The address of a host array (a CPU torch tensor or a C-contiguous numpy array)."""
    if hasattr(p, "data_ptr"):
        if getattr(p, "is_cuda", False):
            raise Error("kernite_b200", "a host array was expected, got a CUDA tensor")
        return int(p.data_ptr())
    if hasattr(p, "ctypes"):
        if not p.flags["C_CONTIGUOUS"]:
            raise Error("kernite_b200", "host arrays must be C-contiguous")
        return int(p.ctypes.data)
    raise TypeError(f"not a host array: {type(p)!r}")


def _stream(s: Any) -> int | None:
    if s is None:
        return None
    if isinstance(s, int):
        return s or None
    if hasattr(s, "cuda_stream"):
        return int(s.cuda_stream) or None
    raise TypeError(f"not a stream: {type(s)!r}")


def module_image() -> bytes:
    """The warp-MMA kernels' sm_100a cubin (``kq_module_image``), for a caller that loads the
    module itself (cuModuleLoadData) and launches what :meth:`Kernels.matvec_plan` plans."""
    p, n = ctypes.c_void_p(), ctypes.c_size_t()
    _check(lib().kq_module_image(ctypes.byref(p), ctypes.byref(n)), "kq_module_image")
    return ctypes.string_at(p.value, n.value)


def stream_key(seed: int, tensor: int) -> int:
    """The stream key of synthetic tensor ``tensor`` under ``seed`` (as the oracle's)."""
    return int(lib().kq_stream_key(seed & (2**64 - 1), tensor & (2**64 - 1)))


class Cuda:
    """GPU ``index``, opened: ``kernite_cuda::Cuda::on(index)``."""

    def __init__(self, index: int = 0):
        self.index = index

    @classmethod
    def on(cls, index: int) -> "Cuda":
        return cls(index)

    @classmethod
    def new(cls) -> "Cuda":
        return cls(0)


class Kernels:
    """The library's kernels loaded on one GPU; one launcher per kernel.

    Every launcher is asynchronous on ``stream`` (None = the legacy default stream, where
    kernite launches) and has kernite's launcher contract: pointers are device memory of this
    GPU, valid and untouched by the host until the launch completes."""

    def __init__(self, ctx: int, cuda: Cuda):
        self._ctx = ctypes.c_void_p(ctx)
        self.cuda = cuda
        dev, sms, smem = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _check(lib().kq_ctx_info(self._ctx, ctypes.byref(dev), ctypes.byref(sms), ctypes.byref(smem)),
               "kq_ctx_info")
        self.device, self.sm_count, self.max_shared = dev.value, sms.value, smem.value

    @classmethod
    def load(cls, cuda: Cuda | int = 0) -> "Kernels":
        if isinstance(cuda, int):
            cuda = Cuda.on(cuda)
        ctx = ctypes.c_void_p()
        _check(lib().kq_ctx_create(cuda.index, ctypes.byref(ctx)), "kq_ctx_create")
        return cls(ctx.value, cuda)

    def close(self) -> None:
        if self._ctx:
            lib().kq_ctx_destroy(self._ctx)
            self._ctx = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self) -> int:
        return int(self._ctx.value or 0)

    # ----------------------------------------------------------------- launchers

    def matvec_q4k(self, y, w, x, rows: int, k: int, batch: int = 1, stream=None) -> None:
        """``y[b*rows + r] = sum_k W[r,k] x[b*k + k]``, W in Q4_K blocks."""
        _check(lib().kq_matvec_q4k(self._ctx, _addr(y), _addr(w), _addr(x), rows, k, batch,
                                   _stream(stream)), "kq_matvec_q4k")

    def matvec_q6k(self, y, w, x, rows: int, k: int, batch: int = 1, stream=None) -> None:
        """The same for Q6_K blocks."""
        _check(lib().kq_matvec_q6k(self._ctx, _addr(y), _addr(w), _addr(x), rows, k, batch,
                                   _stream(stream)), "kq_matvec_q6k")

    def matvec(self, qtype: int, y, w, x, rows: int, k: int, batch: int = 1, *, ldx: int = 0,
               ldy: int = 0, prologue: int = PROLOGUE_NONE, epilogue: int = EPILOGUE_NONE,
               eps: float = 0.0, pair_scale: float = 1.0, flags: int = 0, stream=None) -> None:
        """The general matvec (``kq_matvec``); qtype is 4/5/6 or TYPE_Q4_K/TYPE_Q5_K/TYPE_Q6_K
        (Q5_K at batch 1 only)."""
        t = {2: TYPE_Q2_K, 3: TYPE_Q3_K, 4: TYPE_Q4_K, 5: TYPE_Q5_K, 6: TYPE_Q6_K, 8: TYPE_Q8_0}.get(qtype, qtype)
        d = KqMatvecDesc(type=t, rows=rows, k=k, batch=batch, y=_addr(y), w=_addr(w), x=_addr(x),
                         ldx=ldx, ldy=ldy, prologue=prologue, epilogue=epilogue, eps=eps,
                         pair_scale=pair_scale, flags=flags, reserved=0)
        _check(lib().kq_matvec(self._ctx, ctypes.byref(d), _stream(stream)), "kq_matvec")

    def matvec_host(self, qtype: int, y, w, x, rows: int, k: int, batch: int = 1, *,
                    ldx: int = 0, ldy: int = 0, prologue: int = PROLOGUE_NONE,
                    epilogue: int = EPILOGUE_NONE, eps: float = 0.0, pair_scale: float = 1.0,
                    flags: int = 0, stream=None) -> None:
        """``kq_matvec_host``: x and y are host arrays (torch CPU tensors, pinned for asynchronous
        copies, or numpy arrays), w is on the device; synchronise ``stream`` before reading y."""
        t = {2: TYPE_Q2_K, 3: TYPE_Q3_K, 4: TYPE_Q4_K, 5: TYPE_Q5_K, 6: TYPE_Q6_K, 8: TYPE_Q8_0}.get(qtype, qtype)
        d = KqMatvecDesc(type=t, rows=rows, k=k, batch=batch, y=0, w=_addr(w), x=0, ldx=ldx,
                         ldy=ldy, prologue=prologue, epilogue=epilogue, eps=eps,
                         pair_scale=pair_scale, flags=flags, reserved=0)
        _check(lib().kq_matvec_host(self._ctx, ctypes.byref(d), _host_addr(y), _host_addr(x),
                                    _stream(stream)), "kq_matvec_host")

    def dequant(self, qtype: int, out, w, nblocks: int, stream=None) -> None:
        """Bit-exact decode of ``nblocks`` blocks (units of 256 weights) into f32 (verification
        kernel)."""
        L = lib()
        fn = {2: L.kq_dequant_q2k, 3: L.kq_dequant_q3k, 4: L.kq_dequant_q4k, 5: L.kq_dequant_q5k,
              6: L.kq_dequant_q6k, 8: L.kq_dequant_q8_0}[_qt(qtype)]
        _check(fn(self._ctx, _addr(out), _addr(w), nblocks, _stream(stream)), "kq_dequant")

    def fill(self, qtype: int, w, block0: int, nblocks: int, key: int, stream=None) -> None:
        """Synthetic blocks [block0, block0 + nblocks) of the keyed tensor, written at w."""
        fn = {4: lib().kq_fill_q4k, 5: lib().kq_fill_q5k, 6: lib().kq_fill_q6k}[_qt(qtype)]
        _check(fn(self._ctx, _addr(w), block0, nblocks, key & (2**64 - 1), _stream(stream)), "kq_fill")

    def matvec_q4k_noalloc(self, y, w, x, rows: int, k: int, batch: int = 1, stream=None) -> None:
        """The tensor-core Q4_K matvec without any device allocation (static scratch); see
        ``kq_matvec_q4k_noalloc`` in include/kq.h. Uses the current device."""
        _check(lib().kq_matvec_q4k_noalloc(_addr(y), _addr(w), _addr(x), rows, k, batch,
                                           _stream(stream)), "kq_matvec_q4k_noalloc")

    def matvec_push(self, qtype: int, y, w, x, rows: int, k: int, push: "KqPushDesc", *,
                    prologue: int = PROLOGUE_NONE, epilogue: int = EPILOGUE_NONE, eps: float = 0.0,
                    pair_scale: float = 1.0, flags: int = 0, stream=None) -> None:
        """Batch-1 matvec whose epilogue also stores rows [0, push.push_rows) into every rank's
        full vector and counts them there (``kq_matvec_push``)."""
        t = {2: TYPE_Q2_K, 3: TYPE_Q3_K, 4: TYPE_Q4_K, 5: TYPE_Q5_K, 6: TYPE_Q6_K, 8: TYPE_Q8_0}.get(qtype, qtype)
        d = KqMatvecDesc(type=t, rows=rows, k=k, batch=1, y=_addr(y), w=_addr(w), x=_addr(x),
                         ldx=0, ldy=0, prologue=prologue, epilogue=epilogue, eps=eps,
                         pair_scale=pair_scale, flags=flags, reserved=0)
        _check(lib().kq_matvec_push(self._ctx, ctypes.byref(d), ctypes.byref(push), _stream(stream)),
               "kq_matvec_push")

    def wait_counter(self, counter: int, epoch: int, wait_mul: int, wait_add: int, stream=None) -> None:
        """Stream-ordered bounded wait until *counter >= (*epoch - 1) * wait_mul + wait_add."""
        _check(lib().kq_wait_counter(self._ctx, counter, epoch, wait_mul, wait_add, _stream(stream)),
               "kq_wait_counter")

    def matvec_plan(self, qtype: int, y, w, x, rows: int, k: int, batch: int = 1, *,
                    prologue: int = PROLOGUE_NONE, epilogue: int = EPILOGUE_NONE, eps: float = 0.0,
                    pair_scale: float = 1.0, flags: int = 0) -> "KqLaunch":
        """``kq_matvec_plan``: the warp-MMA launch of this matvec, unlaunched (a function of
        :func:`module_image`, its grid, block, shared memory and parameter bytes)."""
        t = {2: TYPE_Q2_K, 3: TYPE_Q3_K, 4: TYPE_Q4_K, 5: TYPE_Q5_K, 6: TYPE_Q6_K, 8: TYPE_Q8_0}.get(qtype, qtype)
        d = KqMatvecDesc(type=t, rows=rows, k=k, batch=batch, y=_addr(y), w=_addr(w), x=_addr(x),
                         ldx=0, ldy=0, prologue=prologue, epilogue=epilogue, eps=eps,
                         pair_scale=pair_scale, flags=flags, reserved=0)
        out = KqLaunch()
        _check(lib().kq_matvec_plan(self._ctx, ctypes.byref(d), ctypes.byref(out)), "kq_matvec_plan")
        return out

    def rope_append(self, qkv, q_out, k_cache, v_cache, n_heads: int, n_kv: int, head_dim: int,
                    pos: int, base: float = 10000.0, stream=None) -> None:
        """``kq_rope_append``: q rotated into q_out; k rotated and v into row ``pos`` of the f16
        caches."""
        _check(lib().kq_rope_append(self._ctx, _addr(qkv), _addr(q_out), _addr(k_cache), _addr(v_cache),
                                    n_heads, n_kv, head_dim, pos, base, _stream(stream)), "kq_rope_append")

    def attention_workspace(self, n_heads: int, n_kv: int, head_dim: int, length: int) -> int:
        return int(lib().kq_attention_workspace(self._ctx, n_heads, n_kv, head_dim, length))

    def attention(self, out, q, k_cache, v_cache, n_heads: int, n_kv: int, head_dim: int,
                  length: int, workspace, workspace_bytes: int, stream=None) -> None:
        """``kq_attention_decode``: one step's grouped-query attention over the caches' first
        ``length`` positions."""
        _check(lib().kq_attention_decode(self._ctx, _addr(out), _addr(q), _addr(k_cache), _addr(v_cache),
                                         n_heads, n_kv, head_dim, length, _addr(workspace),
                                         workspace_bytes, _stream(stream)), "kq_attention_decode")

    def matvec_chain(self, jobs, epoch: int, stream=None) -> None:
        """``kq_matvec_chain``: up to 8 batch-1 matvecs of one type and k in one launch, each
        waiting for its counter before it reads x (see include/kq.h). ``jobs`` is a sequence of
        :class:`KqChainJob` or a ctypes array of them; ``epoch`` the address of this GPU's u64
        step counter."""
        if not isinstance(jobs, ctypes.Array):
            arr = (KqChainJob * len(jobs))(*jobs)
        else:
            arr = jobs
        _check(lib().kq_matvec_chain(self._ctx, arr, len(arr), epoch, _stream(stream)),
               "kq_matvec_chain")

    def epoch_advance(self, epoch: int, stream=None) -> None:
        """``*epoch += 1`` on the stream: the start of a step for the chains after it."""
        _check(lib().kq_epoch_advance(self._ctx, epoch, _stream(stream)), "kq_epoch_advance")

    def tagged_unpack(self, dst, src, n: int, epoch: int, wait_mul: int, wait_add: int, stream=None) -> None:
        """``kq_tagged_unpack``: the values of a tagged full vector into plain f32, once every
        element carries this step's tag."""
        _check(lib().kq_tagged_unpack(self._ctx, _addr(dst), _addr(src), n, epoch, wait_mul, wait_add,
                                      _stream(stream)), "kq_tagged_unpack")

    def peer_alloc(self, nbytes: int) -> tuple[int, bytes]:
        """Zeroed device memory other GPUs can map; returns (address, 64-byte IPC handle)."""
        ptr = ctypes.c_uint64()
        h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        _check(lib().kq_peer_alloc(self._ctx, nbytes, ctypes.byref(ptr), h), "kq_peer_alloc")
        return ptr.value, h.raw

    def peer_open(self, handle: bytes) -> int:
        ptr = ctypes.c_uint64()
        _check(lib().kq_peer_open(self._ctx, handle, ctypes.byref(ptr)), "kq_peer_open")
        return ptr.value

    def peer_close(self, ptr: int) -> None:
        _check(lib().kq_peer_close(self._ctx, ptr), "kq_peer_close")

    def peer_free(self, ptr: int) -> None:
        _check(lib().kq_peer_free(self._ctx, ptr), "kq_peer_free")

    def device_error(self) -> None:
        """Synchronises the GPU and raises if a kernel's bounded wait gave up."""
        _check(lib().kq_device_error(self._ctx), "kq_device_error")


class DeviceArray:
    """A view of raw device memory that torch (and others) can wrap without a copy through
    ``__cuda_array_interface__``: ``torch.as_tensor(DeviceArray(ptr, n), device="cuda")``."""

    def __init__(self, ptr: int, n: int, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


def _qt(qtype: int) -> int:
    """The type's bit width (2..6; 8 for Q8_0) for a type given that way or by its GGML number
    (10..14, 8)."""
    return {TYPE_Q2_K: 2, TYPE_Q3_K: 3, TYPE_Q4_K: 4, TYPE_Q5_K: 5, TYPE_Q6_K: 6}.get(qtype, qtype)


def block_bytes(qtype: int) -> int:
    """Bytes per 256 weights (a super-block; for Q8_0 eight blocks)."""
    return {2: Q2K_BYTES, 3: Q3K_BYTES, 4: Q4K_BYTES, 5: Q5K_BYTES, 6: Q6K_BYTES,
            8: Q8_0_UNIT_BYTES}[_qt(qtype)]


def matrix_bytes(qtype: int, rows: int, k: int) -> int:
    return rows * (k // QK) * block_bytes(qtype)
