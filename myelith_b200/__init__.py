"""myelith_b200 — B200-native W8A16 integer linear layer for Myelith.

Host-side mirror of the reference's operator interface for this path, over
the C ABI of ``libmyl_w8a16.so`` (include/myl_w8a16.h):

  linear_w8a16(x, W, in_features, w_shifts, act_frac_bits, out_frac_bits)
      INTEGER_LLM/kernels/src/linear.rs:43
  linear_w8a16_pc(x, W, in_features, w_shifts, act_frac_bits, out_frac_bits)
      linear.rs:87
  lm_head_w8a16_i32(x, W, in_features, w_shifts, final_norm_frac, logit_frac)
      runtime/src/model.rs:297-307 (LM head, path B)
  CudaBackend.init(device_id) / .linear_w8a16(x, W, out, in_features,
      out_features, w_shifts, act_frac, out_frac)
      kernels/src/backends/cuda.rs:93, backend.rs:39-49

Arguments have the reference's names and meanings; where the reference
panics (shape assert, debug-build integer overflow) these raise
``MylError`` with the library's status code. Inputs are numpy arrays (one row
[K] or a batch [M, K]; every row gives the reference's per-token result).

The device path (``Context``, ``Weight``, ``Requant`` with torch CUDA tensors)
is what the runtime, the tensor-parallel layer and the benchmark use.

There is no CPU fallback: importing works anywhere, but every compute call
needs the built library and an sm_100 GPU and raises otherwise.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmyl_w8a16.so")

MYL_OK = 0
MYL_ERR_SHAPE = 1
MYL_ERR_OVERFLOW = 2
MYL_ERR_CUDA = 3
MYL_ERR_ARG = 4
MYL_ERR_DEVICE = 5
MYL_ERR_UNSUPPORTED = 6
MYL_ERR_IO = 7
MYL_ERR_CORRUPT = 8

RQ_SHIFT_I16 = 0
RQ_SHIFT_I32 = 1
RQ_MULT_I16 = 2

_STATUS = {1: "shape", 2: "overflow", 3: "cuda", 4: "argument", 5: "device", 6: "unsupported",
           7: "io", 8: "corrupt"}


class MylError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn}: {_STATUS.get(code, 'error')} error ({code}): {msg}")
        self.code = code


_lib = None
_lib_lock = threading.Lock()


def load_library(path: str | None = None):
    """Loads libmyl_w8a16.so (raises if it is missing: there is no fallback)."""
    global _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise MylError("load_library", MYL_ERR_UNSUPPORTED,
                           f"{p} is missing; build it with `python -m myelith_b200.build`")
        L = C.CDLL(p)
        vp, i64, u8, i32 = C.c_void_p, C.c_int64, C.c_uint8, C.c_int
        sig = {
            "myl_last_error": ([], C.c_char_p),
            "myl_abi_version": ([], i32),
            "myl_init": ([i32, C.POINTER(vp)], i32),
            "myl_destroy": ([vp], i32),
            "myl_device_info": ([vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32)], i32),
            "myl_weight_register": ([vp, vp, i64, i64, i64, vp, C.POINTER(vp)], i32),
            "myl_weight_release": ([vp, vp], i32),
            "myl_linear_w8a16": ([vp, vp, vp, i64, u8, u8, vp], i32),
            "myl_linear_w8a16_pc": ([vp, vp, vp, i64, u8, vp, vp], i32),
            "myl_lm_head_w8a16_i32": ([vp, vp, vp, i64, u8, u8, vp], i32),
            "myl_linear_w8a16_mult": ([vp, vp, vp, i64, vp, vp, vp], i32),
            "myl_backend_linear_w8a16": ([vp, vp, vp, vp, C.c_uint64, C.c_uint64, vp, u8, u8], i32),
            "myl_backend_forget": ([vp, vp], i32),
            "myl_requant_create": ([vp, vp, i32, u8, vp, i32, vp, vp, C.POINTER(vp)], i32),
            "myl_requant_release": ([vp, vp], i32),
            "myl_linear_dev": ([vp, vp, vp, vp, i64, i64, vp, i64, vp], i32),
            "myl_linear_acc_dev": ([vp, vp, vp, i64, i64, vp, vp], i32),
            "myl_requant_acc_dev": ([vp, vp, vp, i64, vp, i64, vp], i32),
            "myl_split_hilo_dev": ([vp, vp, i64, i64, i64, vp, vp, i64, vp], i32),
            "myl_linear_planes_dev": ([vp, vp, vp, vp, vp, i64, i64, vp, i64, vp], i32),
            "myl_linear_w8a16_bias": ([vp, vp, vp, i64, u8, u8, vp, vp, vp], i32),
            "myl_requant_set_bias": ([vp, vp, vp, vp, u8], i32),
            "myl_mlp_register": ([vp, vp, vp, vp, i64, i64, vp, vp, vp, vp, i64, u8, u8, u8, u8, u8,
                                  C.c_int16, u8, vp, C.POINTER(vp)], i32),
            "myl_mlp_release": ([vp, vp], i32),
            "myl_mlp_int": ([vp, vp, vp, i64, vp], i32),
            "myl_mlp_dev": ([vp, vp, vp, i64, i64, vp, i64, vp], i32),
            "myl_mlp_partial_dev": ([vp, vp, vp, i64, i64, vp, vp], i32),
            "myl_mlp_requant_dev": ([vp, vp, vp, i64, vp, i64, vp], i32),
            "myl_synchronize": ([vp], i32),
            "myl_set_wait_timeout_ns": ([vp, C.c_uint64], i32),
            "myl_set_dispatch": ([vp, i32, i32, i32], i32),
            "myl_launch_count": ([vp], i64),
            "myl_set_sm_limit": ([vp, i32], i32),
            "myl_set_tc_options": ([vp, i32, i32], i32),
            "myl_argmax_keys_dev": ([vp, vp, i64, i64, i64, i64, vp, vp], i32),
            "myl_linear_acc_exchange_dev": ([vp, vp, vp, i64, i64, vp, i32, i32, i64, vp], i32),
            "myl_exchange_reduce_dev": ([vp, vp, vp, i32, i32, i64, i64, vp, i64, vp], i32),
            "myl_exchange_barrier_dev": ([vp, vp, i32, i32, C.c_uint64, vp], i32),
            "myl_ep_dispatch_dev": ([vp, vp, i64, i64, i64, vp, i32, i32, i32, i32, vp, vp, vp, vp,
                                     i64, vp], i32),
            "myl_ep_return_dev": ([vp, vp, i64, i64, vp, vp, i32, vp], i32),
            "myl_ipc_alloc": ([vp, C.c_size_t, C.POINTER(vp), vp], i32),
            "myl_ipc_open": ([vp, vp, C.POINTER(vp)], i32),
            "myl_ipc_close": ([vp, vp], i32),
            "myl_ipc_free": ([vp, vp], i32),
            "myl_wire_frame_bytes": ([C.c_uint64], C.c_uint64),
            "myl_crc32": ([vp, C.c_uint64], C.c_uint32),
            "myl_wire_encode": ([vp, vp, C.c_uint64, vp, C.c_uint64, C.POINTER(C.c_uint64)], i32),
            "myl_wire_decode": ([vp, C.c_uint64, vp, vp, C.c_uint64, C.POINTER(C.c_uint64)], i32),
            "myl_crc32_dev": ([vp, vp, C.c_uint64, C.POINTER(C.c_uint32), vp], i32),
            "myl_wire_decode_dev": ([vp, vp, C.c_uint64, vp, vp, C.c_uint64, C.POINTER(C.c_uint64), vp], i32),
            "myl_wire_encode_dev": ([vp, vp, vp, C.c_uint64, vp, C.c_uint64, C.POINTER(C.c_uint64), vp], i32),
            "myl_wire_pack_tokens": ([vp, C.c_uint64, vp], i32),
            "myl_wire_unpack_tokens": ([vp, C.c_uint64, vp], i32),
            "myl_debug_inject_wait_fault": ([vp, i32], i32),
            "myl_weight16_register": ([vp, vp, i64, i64, i64, vp, C.POINTER(vp)], i32),
            "myl_linear_backward": ([vp, vp, vp, vp, i64, u8, u8, vp, vp], i32),
            "myl_linear_backward_dev": ([vp, vp, vp, i64, vp, i64, i64, u8, u8, vp, i64, vp, vp], i32),
            "myl_lm_head_w16a16_i32": ([vp, vp, vp, i64, u8, u8, vp], i32),
            "myl_sha256": ([vp, C.c_size_t, vp], i32),
            "myl_artifact_open": ([C.c_char_p, C.POINTER(vp)], i32),
            "myl_artifact_close": ([vp], i32),
            "myl_artifact_count": ([vp], i64),
            "myl_artifact_find": ([vp, C.c_char_p, C.POINTER(i64)], i32),
            "myl_artifact_tensor": ([vp, i64, C.POINTER(C.c_char_p), C.POINTER(C.c_char_p),
                                     C.POINTER(i32), C.POINTER(i32), C.POINTER(i64), C.POINTER(vp),
                                     C.POINTER(vp)], i32),
            "myl_artifact_register": ([vp, vp, i64, C.POINTER(vp)], i32),
            "myl_artifact_lut": ([vp, C.c_char_p, C.POINTER(vp), C.POINTER(i64)], i32),
            "myl_moe_register": ([vp, C.POINTER(MoeSpec), C.POINTER(vp)], i32),
            "myl_moe_release": ([vp, vp], i32),
            "myl_moe_forward": ([vp, vp, vp, i64, vp], i32),
            "myl_moe_dev": ([vp, vp, vp, i64, i64, vp, i64, vp, vp, vp], i32),
            "myl_moe_route_dev": ([vp, vp, vp, i64, i64, vp, vp, vp], i32),
            "myl_moe_experts_dev": ([vp, vp, vp, i64, i64, vp, vp, i64, vp], i32),
            "myl_moe_combine_dev": ([vp, vp, vp, i64, vp, vp, i64, i64, vp, i64, vp], i32),
        }
        for name, (args, res) in sig.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
        return L


def _check(fn: str, rc: int) -> None:
    if rc != MYL_OK:
        msg = load_library().myl_last_error().decode(errors="replace")
        raise MylError(fn, rc, msg)


def _p(a) -> int | None:
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return int(a.data_ptr())  # torch tensor


def _c(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=dtype))


class Context:
    """One device context (CudaBackend::init, kernels/src/backends/cuda.rs:93)."""

    def __init__(self, device: int = 0):
        L = load_library()
        h = C.c_void_p()
        _check("myl_init", L.myl_init(device, C.byref(h)))
        self._h = h
        self.device = device
        d, sm, nsm = C.c_int(), C.c_int(), C.c_int()
        _check("myl_device_info", L.myl_device_info(h, C.byref(d), C.byref(sm), C.byref(nsm)))
        self.sm_version = sm.value
        self.num_sms = nsm.value

    @property
    def handle(self):
        return self._h

    def close(self) -> None:
        if getattr(self, "_h", None):
            load_library().myl_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def synchronize(self) -> None:
        _check("myl_synchronize", load_library().myl_synchronize(self._h))

    def set_wait_timeout_ns(self, ns: int) -> None:
        _check("myl_set_wait_timeout_ns", load_library().myl_set_wait_timeout_ns(self._h, ns))

    def set_dispatch(self, gemv_max_m: int = 4, force_split_k: int = 0, force_token_tile: int = 0) -> None:
        _check("myl_set_dispatch",
               load_library().myl_set_dispatch(self._h, gemv_max_m, force_split_k, force_token_tile))

    def set_sm_limit(self, max_sms: int) -> None:
        """Persistent kernels use at most max_sms SMs (0: all)."""
        _check("myl_set_sm_limit", load_library().myl_set_sm_limit(self._h, max_sms))

    def ipc_alloc(self, nbytes: int) -> tuple[int, bytes]:
        """Device buffer shareable with the other processes of the node:
        (device pointer, IPC handle bytes)."""
        ptr = C.c_void_p()
        h = (C.c_uint8 * IPC_HANDLE_BYTES)()
        _check("myl_ipc_alloc", load_library().myl_ipc_alloc(self._h, nbytes, C.byref(ptr), h))
        return int(ptr.value), bytes(h)

    def ipc_open(self, handle: bytes) -> int:
        """Maps another process's buffer (its IPC handle) into this one."""
        ptr = C.c_void_p()
        h = (C.c_uint8 * IPC_HANDLE_BYTES).from_buffer_copy(handle)
        _check("myl_ipc_open", load_library().myl_ipc_open(self._h, h, C.byref(ptr)))
        return int(ptr.value)

    def exchange_barrier_dev(self, flag_ptrs, rank: int, epoch: int, stream=None) -> None:
        """Device-side barrier of a peer-memory exchange (myl_exchange_barrier_dev)."""
        arr = (C.c_void_p * len(flag_ptrs))(*flag_ptrs)
        _check("myl_exchange_barrier_dev", load_library().myl_exchange_barrier_dev(
            self._h, arr, len(flag_ptrs), rank, epoch, _stream_ptr(stream)))

    def ep_dispatch_dev(self, x, idx, num_experts: int, rank: int, rows, ids, src, counters,
                        capacity: int, stream=None) -> None:
        """Expert-parallel dispatch over peer memory (myl_ep_dispatch_dev); rows,
        ids, src, counters: one device pointer per rank."""
        w = len(rows)
        arr = [(C.c_void_p * w)(*a) for a in (rows, ids, src, counters)]
        _check("myl_ep_dispatch_dev", load_library().myl_ep_dispatch_dev(
            self._h, _p(x), x.shape[0], x.stride(0), x.shape[1], _p(idx), idx.shape[1], num_experts,
            w, rank, arr[0], arr[1], arr[2], arr[3], capacity, _stream_ptr(stream)))

    def ep_return_dev(self, y, count: int, src, back, stream=None) -> None:
        """Returns received expert outputs to their home ranks (myl_ep_return_dev)."""
        arr = (C.c_void_p * len(back))(*back)
        _check("myl_ep_return_dev", load_library().myl_ep_return_dev(
            self._h, _p(y), count, y.shape[1], _p(src), arr, len(back), _stream_ptr(stream)))

    def ipc_close(self, ptr: int) -> None:
        _check("myl_ipc_close", load_library().myl_ipc_close(self._h, C.c_void_p(ptr)))

    def ipc_free(self, ptr: int) -> None:
        _check("myl_ipc_free", load_library().myl_ipc_free(self._h, C.c_void_p(ptr)))

    def crc32_dev(self, data, stream=None) -> int:
        """CRC-32 (crc32fast / zlib) of a torch CUDA tensor's bytes, on the GPU."""
        out = C.c_uint32()
        _check("myl_crc32_dev", load_library().myl_crc32_dev(
            self._h, _p(data), data.numel() * data.element_size(), C.byref(out), _stream_ptr(stream)))
        return out.value

    def wire_decode_dev(self, frame: bytes, values, stream=None) -> tuple[dict, int]:
        """Decodes an IINTPIPE frame into the int16 CUDA tensor values (payload
        CRC checked on the GPU); returns (meta, number of values)."""
        m = WireMeta()
        n = C.c_uint64()
        buf = np.frombuffer(frame, np.uint8)
        _check("myl_wire_decode_dev", load_library().myl_wire_decode_dev(
            self._h, _p(buf), buf.size, C.byref(m), _p(values), values.numel(), C.byref(n),
            _stream_ptr(stream)))
        return m.as_dict(), n.value

    def wire_encode_dev(self, meta: dict, values, stream=None) -> bytes:
        """IINTPIPE frame of the int16 CUDA tensor values (CRC on the GPU)."""
        n = values.numel()
        out = np.zeros(load_library().myl_wire_frame_bytes(n), np.uint8)
        ln = C.c_uint64()
        m = WireMeta.from_dict(meta)
        _check("myl_wire_encode_dev", load_library().myl_wire_encode_dev(
            self._h, C.byref(m), _p(values), n, _p(out), out.size, C.byref(ln), _stream_ptr(stream)))
        return out[: ln.value].tobytes()

    def argmax_keys_dev(self, logits, keys, index_base: int = 0, stream=None) -> None:
        """keys[M] int64 = greedy selection keys of int32 logits [M, V] (torch
        CUDA tensors) whose column j is vocab index index_base + j; see
        keys_to_tokens."""
        M, V = (logits.shape[0], logits.shape[1]) if logits.dim() == 2 else (1, logits.shape[0])
        ld = logits.stride(0) if logits.dim() == 2 else V
        _check("myl_argmax_keys_dev", load_library().myl_argmax_keys_dev(
            self._h, _p(logits), M, V, ld, index_base, _p(keys), _stream_ptr(stream)))

    def set_tc_options(self, pair: bool = True, xbox_rows: int = 0) -> None:
        """Tensor-core GEMM variant: CTA pairs for 128-token tiles (default) or
        one CTA per tile; activation TMA box height (0 = unchanged)."""
        _check("myl_set_tc_options",
               load_library().myl_set_tc_options(self._h, 1 if pair else 0, xbox_rows))

    def inject_wait_fault(self, on: bool) -> None:
        _check("myl_debug_inject_wait_fault",
               load_library().myl_debug_inject_wait_fault(self._h, 1 if on else 0))

    @property
    def launch_count(self) -> int:
        return int(load_library().myl_launch_count(self._h))

    def weight(self, W, in_features: int, w_shifts, ldw: int | None = None) -> "Weight":
        return Weight(self, W, in_features, w_shifts, ldw)

    def weight16(self, W, in_features: int, w_shifts) -> "Weight16":
        return Weight16(self, W, in_features, w_shifts)

    def split_hilo_dev(self, x, xhi, xlo, stream=None) -> None:
        """x [M, K] int16 (torch CUDA) -> byte planes xhi int8 / xlo uint8 [M, ldp]."""
        M, K = x.shape
        _check("myl_split_hilo_dev", load_library().myl_split_hilo_dev(
            self._h, _p(x), M, K, x.stride(0), _p(xhi), _p(xlo), xhi.stride(0), _stream_ptr(stream)))


class Weight:
    """A weight matrix uploaded once ([out_features][in_features] int8 plus
    one power-of-two shift per output row, runtime/src/model.rs:28-35)."""

    def __init__(self, ctx: Context, W, in_features: int, w_shifts, ldw: int | None = None):
        self.ctx = ctx
        w_shifts = _c(w_shifts, np.uint8)
        W = np.asarray(W, dtype=np.int8)
        if W.ndim == 2 and ldw is None:
            ldw = W.shape[1]
            W = np.ascontiguousarray(W)
        ldw = in_features if ldw is None else ldw
        W = np.ascontiguousarray(W).reshape(-1)
        N = w_shifts.size
        if in_features <= 0 or ldw < in_features or (N > 0 and W.size < (N - 1) * ldw + in_features):
            raise MylError("myl_weight_register", MYL_ERR_SHAPE,
                           f"{W.size} weights do not hold {N} rows of {in_features}")
        h = C.c_void_p()
        _check("myl_weight_register", load_library().myl_weight_register(
            ctx.handle, _p(W), N, in_features, ldw, _p(w_shifts), C.byref(h)))
        self._h = h
        self.out_features = N
        self.in_features = in_features
        self.w_shifts = w_shifts

    @property
    def handle(self):
        return self._h

    def release(self) -> None:
        if getattr(self, "_h", None) and self.ctx.handle:
            load_library().myl_weight_release(self.ctx.handle, self._h)
        self._h = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    # ---- host-pointer calls (synchronous) ----
    def _rows(self, x):
        x = _c(x, np.int16)
        single = x.ndim == 1
        xs = x.reshape(1, -1) if single else x
        if xs.shape[1] != self.in_features:
            raise MylError("linear", MYL_ERR_SHAPE,
                           f"x rows have {xs.shape[1]} elements, weight expects {self.in_features}")
        return np.ascontiguousarray(xs), single

    def linear(self, x, act_frac_bits: int, out_frac_bits) -> np.ndarray:
        """linear_w8a16 (scalar out_frac) or linear_w8a16_pc (array out_frac)."""
        xs, single = self._rows(x)
        y = np.zeros((xs.shape[0], self.out_features), np.int16)
        L = load_library()
        if np.ndim(out_frac_bits) == 0:
            _check("myl_linear_w8a16", L.myl_linear_w8a16(
                self.ctx.handle, self._h, _p(xs), xs.shape[0], act_frac_bits, int(out_frac_bits), _p(y)))
        else:
            of = _c(out_frac_bits, np.uint8)
            if of.size != self.out_features:
                raise MylError("myl_linear_w8a16_pc", MYL_ERR_SHAPE, "one out_frac per channel")
            _check("myl_linear_w8a16_pc", L.myl_linear_w8a16_pc(
                self.ctx.handle, self._h, _p(xs), xs.shape[0], act_frac_bits, _p(of), _p(y)))
        return y[0] if single else y

    def lm_head(self, x, final_norm_frac: int, logit_frac: int) -> np.ndarray:
        xs, single = self._rows(x)
        y = np.zeros((xs.shape[0], self.out_features), np.int32)
        _check("myl_lm_head_w8a16_i32", load_library().myl_lm_head_w8a16_i32(
            self.ctx.handle, self._h, _p(xs), xs.shape[0], final_norm_frac, logit_frac, _p(y)))
        return y[0] if single else y

    def linear_bias(self, x, act_frac_bits: int, out_frac_bits: int, bias, bias_shifts) -> np.ndarray:
        """linear_w8a16 then add_bias_i16, fused (runtime/src/model.rs:438-453)."""
        xs, single = self._rows(x)
        b = _c(bias, np.int16)
        bs = _c(bias_shifts, np.uint8)
        if b.size != self.out_features or bs.size != self.out_features:
            raise MylError("add_bias_i16", MYL_ERR_SHAPE, "one bias and shift per channel")
        y = np.zeros((xs.shape[0], self.out_features), np.int16)
        _check("myl_linear_w8a16_bias", load_library().myl_linear_w8a16_bias(
            self.ctx.handle, self._h, _p(xs), xs.shape[0], act_frac_bits, out_frac_bits, _p(b), _p(bs),
            _p(y)))
        return y[0] if single else y

    def linear_mult(self, x, mult, shift) -> np.ndarray:
        xs, single = self._rows(x)
        mult = _c(mult, np.int32)
        shift = _c(shift, np.uint8)
        if mult.size != self.out_features or shift.size != self.out_features:
            raise MylError("myl_linear_w8a16_mult", MYL_ERR_SHAPE, "one mult/shift per channel")
        y = np.zeros((xs.shape[0], self.out_features), np.int16)
        _check("myl_linear_w8a16_mult", load_library().myl_linear_w8a16_mult(
            self.ctx.handle, self._h, _p(xs), xs.shape[0], _p(mult), _p(shift), _p(y)))
        return y[0] if single else y

    # ---- device path (torch CUDA tensors) ----
    def requant(self, mode: int = RQ_SHIFT_I16, act_frac: int = 0, out_frac=0, mult=None,
                shift=None) -> "Requant":
        return Requant(self, mode, act_frac, out_frac, mult, shift)

    def backward(self, g, x, g_frac: int, gx_frac: int, want_gw: bool = True):
        """linear_backward (kernels/src/backward.rs:147-211) on M tokens:
        g [M, N] int32, x [M, K] int16 -> (gx [M, K] int32, gw [M, N, K] int64 or None)."""
        g = np.ascontiguousarray(_c(g, np.int32).reshape(-1, self.out_features))
        xs = np.ascontiguousarray(_c(x, np.int16).reshape(-1, self.in_features))
        if xs.shape[0] != g.shape[0]:
            raise MylError("myl_linear_backward", MYL_ERR_SHAPE, "g and x have different row counts")
        M = g.shape[0]
        gx = np.zeros((M, self.in_features), np.int32)
        gw = np.zeros((M, self.out_features, self.in_features), np.int64) if want_gw else None
        _check("myl_linear_backward", load_library().myl_linear_backward(
            self.ctx.handle, self._h, _p(g), _p(xs), M, g_frac, gx_frac, _p(gx), _p(gw)))
        return gx, gw

    def backward_dev(self, g, x, g_frac: int, gx_frac: int, gx, gw=None, stream=None) -> None:
        _check("myl_linear_backward_dev", load_library().myl_linear_backward_dev(
            self.ctx.handle, self._h, _p(g), g.stride(0), _p(x), x.stride(0), g.shape[0], g_frac,
            gx_frac, _p(gx), gx.stride(0), _p(gw), _stream_ptr(stream)))

    def linear_dev(self, rq: "Requant", x, y, stream=None) -> None:
        """y[M, N] = requant(W x) for torch CUDA tensors x [M, >=K] int16."""
        M = x.shape[0]
        _check("myl_linear_dev", load_library().myl_linear_dev(
            self.ctx.handle, self._h, rq.handle, _p(x), M, x.stride(0), _p(y), y.stride(0),
            _stream_ptr(stream)))

    def linear_planes_dev(self, rq, xhi, xlo, M: int, y, stream=None) -> None:
        """Tensor-core GEMM from byte planes; rq=None stores int64 accumulators."""
        _check("myl_linear_planes_dev", load_library().myl_linear_planes_dev(
            self.ctx.handle, self._h, None if rq is None else rq.handle, _p(xhi), _p(xlo),
            xhi.stride(0), M, _p(y), y.stride(0), _stream_ptr(stream)))

    def acc_exchange_dev(self, x, dst_ptrs, rank: int, rows_per_rank: int, stream=None) -> None:
        """Exact int64 partials of W x stored into the owning ranks' receive
        buffers (myl_linear_acc_exchange_dev; dst_ptrs: one device pointer per
        rank)."""
        arr = (C.c_void_p * len(dst_ptrs))(*dst_ptrs)
        _check("myl_linear_acc_exchange_dev", load_library().myl_linear_acc_exchange_dev(
            self.ctx.handle, self._h, _p(x), x.shape[0], x.stride(0), arr, len(dst_ptrs), rank,
            rows_per_rank, _stream_ptr(stream)))

    def linear_acc_dev(self, x, acc, stream=None) -> None:
        """acc[M, N] int64 = exact W x (no requant)."""
        _check("myl_linear_acc_dev", load_library().myl_linear_acc_dev(
            self.ctx.handle, self._h, _p(x), x.shape[0], x.stride(0), _p(acc), _stream_ptr(stream)))


class Weight16(Weight):
    """An int16 LM-head weight (runtime/src/loader.rs:124-128: int16 [vocab][hidden]
    plus one shift per row), for path A of the LM head (model.rs:285-296)."""

    def __init__(self, ctx: Context, W, in_features: int, w_shifts):
        self.ctx = ctx
        w_shifts = _c(w_shifts, np.uint8)
        W = np.ascontiguousarray(np.asarray(W, dtype=np.int16)).reshape(-1)
        N = w_shifts.size
        if in_features <= 0 or W.size != N * in_features:
            raise MylError("myl_weight16_register", MYL_ERR_SHAPE,
                           f"{W.size} weights do not hold {N} rows of {in_features}")
        h = C.c_void_p()
        _check("myl_weight16_register", load_library().myl_weight16_register(
            ctx.handle, _p(W), N, in_features, in_features, _p(w_shifts), C.byref(h)))
        self._h = h
        self.out_features = N
        self.in_features = in_features
        self.w_shifts = w_shifts

    def lm_head(self, x, final_norm_frac: int, logit_frac: int) -> np.ndarray:
        """LM head path A: i32 logits [M, vocab]."""
        xs, single = self._rows(x)
        y = np.zeros((xs.shape[0], self.out_features), np.int32)
        _check("myl_lm_head_w16a16_i32", load_library().myl_lm_head_w16a16_i32(
            self.ctx.handle, self._h, _p(xs), xs.shape[0], final_norm_frac, logit_frac, _p(y)))
        return y[0] if single else y


class Requant:
    """Per-channel requant plan kept on the device (myl_requant_create)."""

    def __init__(self, w: Weight, mode: int, act_frac: int, out_frac, mult, shift):
        self.w = w
        per_channel = np.ndim(out_frac) > 0
        of = _c(np.atleast_1d(out_frac), np.uint8)
        m = None if mult is None else _c(mult, np.int32)
        s = None if shift is None else _c(shift, np.uint8)
        h = C.c_void_p()
        _check("myl_requant_create", load_library().myl_requant_create(
            w.ctx.handle, w.handle, mode, act_frac, _p(of), 1 if per_channel else 0, _p(m), _p(s),
            C.byref(h)))
        self._h = h
        self.mode = mode

    def exchange_reduce_dev(self, recv_ptr: int, world: int, rank: int, rows_per_rank: int, M: int,
                            out_ptrs, ldo: int, stream=None) -> None:
        """Sums this rank's slabs of the exchange's receive buffer, requantises
        and writes the rows into every rank's output buffer
        (myl_exchange_reduce_dev)."""
        arr = (C.c_void_p * len(out_ptrs))(*out_ptrs)
        _check("myl_exchange_reduce_dev", load_library().myl_exchange_reduce_dev(
            self.w.ctx.handle, self._h, C.c_void_p(recv_ptr), world, rank, rows_per_rank, M, arr,
            ldo, _stream_ptr(stream)))

    @property
    def handle(self):
        return self._h

    def release(self) -> None:
        if getattr(self, "_h", None):
            load_library().myl_requant_release(self.w.ctx.handle, self._h)
        self._h = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    def set_bias(self, bias, bias_shifts, out_frac: int) -> None:
        b = _c(bias, np.int16)
        bs = _c(bias_shifts, np.uint8)
        _check("myl_requant_set_bias", load_library().myl_requant_set_bias(
            self.w.ctx.handle, self._h, _p(b), _p(bs), out_frac))

    def apply_acc_dev(self, acc, y, stream=None) -> None:
        _check("myl_requant_acc_dev", load_library().myl_requant_acc_dev(
            self.w.ctx.handle, self._h, _p(acc), acc.shape[0], _p(y), y.stride(0),
            _stream_ptr(stream)))


class Mlp:
    """mlp_int (kernels/src/mlp.rs:28-74) with its weights and scales
    registered once (gate/up interleaved on the device)."""

    def __init__(self, ctx: Context, W_gate, W_up, W_down, hidden_size: int, intermediate_size: int,
                 gate_w_shifts, up_w_shifts, down_w_shifts, silu_lut, in_frac_bits: int,
                 gate_out_frac: int, up_out_frac: int, down_in_frac: int, silu_in_frac: int,
                 silu_lut_offset: int, silu_out_frac: int, out_frac_bits):
        H, I = hidden_size, intermediate_size
        Wg, Wu, Wd = (_c(a, np.int8).reshape(-1) for a in (W_gate, W_up, W_down))
        gs, us, ds = (_c(a, np.uint8) for a in (gate_w_shifts, up_w_shifts, down_w_shifts))
        lut = _c(silu_lut, np.int16)
        of = _c(out_frac_bits, np.uint8)
        if (H <= 0 or I <= 0 or Wg.size != H * I or Wu.size != H * I or Wd.size != H * I
                or gs.size != I or us.size != I or ds.size != H or of.size != H):
            raise MylError("mlp_int", MYL_ERR_SHAPE, "weight/shift lengths do not match the shape")
        h = C.c_void_p()
        _check("myl_mlp_register", load_library().myl_mlp_register(
            ctx.handle, _p(Wg), _p(Wu), _p(Wd), H, I, _p(gs), _p(us), _p(ds), _p(lut), lut.size,
            in_frac_bits, gate_out_frac, up_out_frac, down_in_frac, silu_in_frac, silu_lut_offset,
            silu_out_frac, _p(of), C.byref(h)))
        self.ctx, self._h, self.hidden, self.intermediate = ctx, h, H, I

    @property
    def handle(self):
        return self._h

    def release(self) -> None:
        if getattr(self, "_h", None) and self.ctx.handle:
            load_library().myl_mlp_release(self.ctx.handle, self._h)
        self._h = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    def __call__(self, x) -> np.ndarray:
        x = _c(x, np.int16)
        single = x.ndim == 1
        xs = np.ascontiguousarray(x.reshape(1, -1) if single else x)
        if xs.shape[1] != self.hidden:
            raise MylError("mlp_int", MYL_ERR_SHAPE, "x rows must have hidden_size elements")
        y = np.zeros_like(xs)
        _check("myl_mlp_int", load_library().myl_mlp_int(self.ctx.handle, self._h, _p(xs),
                                                           xs.shape[0], _p(y)))
        return y[0] if single else y

    def dev(self, x, y, stream=None) -> None:
        _check("myl_mlp_dev", load_library().myl_mlp_dev(
            self.ctx.handle, self._h, _p(x), x.shape[0], x.stride(0), _p(y), y.stride(0),
            _stream_ptr(stream)))

    def partial_dev(self, x, acc, stream=None) -> None:
        """acc [M, hidden] int64: exact down-projection sums of this slice."""
        _check("myl_mlp_partial_dev", load_library().myl_mlp_partial_dev(
            self.ctx.handle, self._h, _p(x), x.shape[0], x.stride(0), _p(acc), _stream_ptr(stream)))

    def requant_dev(self, acc, y, stream=None) -> None:
        _check("myl_mlp_requant_dev", load_library().myl_mlp_requant_dev(
            self.ctx.handle, self._h, _p(acc), acc.shape[0], _p(y), y.stride(0), _stream_ptr(stream)))


class MoeSpec(C.Structure):
    """myl_moe_spec (include/myl_w8a16.h)."""

    _fields_ = [
        ("hidden", C.c_int64), ("intermediate", C.c_int64), ("num_experts", C.c_int64),
        ("top_k", C.c_int64), ("first_expert", C.c_int64), ("num_local", C.c_int64),
        ("W_router", C.c_void_p), ("router_w_shifts", C.c_void_p),
        ("router_in_frac", C.c_uint8), ("router_frac", C.c_uint8),
        ("exp_lut", C.c_void_p), ("exp_lut_len", C.c_int64),
        ("exp_lut_shift", C.c_uint8), ("prob_frac", C.c_uint8),
        ("W_gate", C.c_void_p), ("W_up", C.c_void_p), ("W_down", C.c_void_p),
        ("gate_w_shifts", C.c_void_p), ("up_w_shifts", C.c_void_p), ("down_w_shifts", C.c_void_p),
        ("out_frac", C.c_void_p),
        ("silu_lut", C.c_void_p), ("silu_lut_len", C.c_int64),
        ("in_frac", C.c_uint8), ("gate_out_frac", C.c_uint8), ("up_out_frac", C.c_uint8),
        ("down_in_frac", C.c_uint8), ("silu_in_frac", C.c_uint8), ("silu_out_frac", C.c_uint8),
        ("silu_lut_offset", C.c_int16),
        ("shared", C.c_void_p),
    ]


class Moe:
    """MoE layer built from the reference's primitives (router = LM-head
    linear, integer top-k with the lowest index winning ties, softmax_int,
    experts = mlp_int, combine = rescale_i64 of the probability-weighted sum
    plus the shared expert). The object holds experts
    [first_expert, first_expert + num_local) of num_experts; the router always
    covers all of them.

    Expert arrays: W_gate / W_up [num_local, I, H], W_down [num_local, H, I],
    gate/up_w_shifts [num_local, I], down_w_shifts / out_frac [num_local, H].
    ``shared`` is an ``Mlp`` (kept alive by this object) or None."""

    def __init__(self, ctx: Context, hidden: int, intermediate: int, num_experts: int, top_k: int,
                 W_router, router_w_shifts, router_in_frac: int, router_frac: int,
                 exp_lut, exp_lut_shift: int, prob_frac: int,
                 W_gate, W_up, W_down, gate_w_shifts, up_w_shifts, down_w_shifts, out_frac,
                 silu_lut, in_frac: int, gate_out_frac: int, up_out_frac: int, down_in_frac: int,
                 silu_in_frac: int, silu_lut_offset: int, silu_out_frac: int,
                 shared: "Mlp | None" = None, first_expert: int = 0, num_local: int | None = None):
        H, I, E = hidden, intermediate, num_experts
        Lc = E if num_local is None else num_local
        arrs = dict(
            W_router=_c(W_router, np.int8).reshape(-1), router_w_shifts=_c(router_w_shifts, np.uint8),
            exp_lut=_c(exp_lut, np.int16).reshape(-1),
            W_gate=_c(W_gate, np.int8).reshape(-1), W_up=_c(W_up, np.int8).reshape(-1),
            W_down=_c(W_down, np.int8).reshape(-1),
            gate_w_shifts=_c(gate_w_shifts, np.uint8).reshape(-1),
            up_w_shifts=_c(up_w_shifts, np.uint8).reshape(-1),
            down_w_shifts=_c(down_w_shifts, np.uint8).reshape(-1),
            out_frac=_c(out_frac, np.uint8).reshape(-1), silu_lut=_c(silu_lut, np.int16).reshape(-1))
        want = dict(W_router=E * H, router_w_shifts=E, W_gate=Lc * I * H, W_up=Lc * I * H,
                    W_down=Lc * H * I, gate_w_shifts=Lc * I, up_w_shifts=Lc * I,
                    down_w_shifts=Lc * H, out_frac=Lc * H)
        for k, n in want.items():
            if arrs[k].size != n:
                raise MylError("moe", MYL_ERR_SHAPE, f"{k} has {arrs[k].size} elements, expected {n}")
        spec = MoeSpec(hidden=H, intermediate=I, num_experts=E, top_k=top_k, first_expert=first_expert,
                       num_local=Lc, router_in_frac=router_in_frac, router_frac=router_frac,
                       exp_lut_len=arrs["exp_lut"].size, exp_lut_shift=exp_lut_shift,
                       prob_frac=prob_frac, silu_lut_len=arrs["silu_lut"].size, in_frac=in_frac,
                       gate_out_frac=gate_out_frac, up_out_frac=up_out_frac,
                       down_in_frac=down_in_frac, silu_in_frac=silu_in_frac,
                       silu_out_frac=silu_out_frac, silu_lut_offset=silu_lut_offset,
                       shared=shared.handle.value if shared is not None else None)
        for k, a in arrs.items():
            setattr(spec, k, _p(a) if a.size else None)
        h = C.c_void_p()
        _check("myl_moe_register", load_library().myl_moe_register(ctx.handle, C.byref(spec), C.byref(h)))
        self.ctx, self._h, self.shared = ctx, h, shared
        self.hidden, self.intermediate, self.num_experts, self.top_k = H, I, E, top_k
        self.first_expert, self.num_local = first_expert, Lc

    @property
    def handle(self):
        return self._h

    def release(self) -> None:
        if getattr(self, "_h", None) and self.ctx.handle:
            load_library().myl_moe_release(self.ctx.handle, self._h)
        self._h = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    def __call__(self, x) -> np.ndarray:
        """Host arrays: x [T, hidden] int16 -> [T, hidden] int16."""
        xs = np.ascontiguousarray(_c(x, np.int16).reshape(-1, self.hidden))
        y = np.zeros_like(xs)
        _check("myl_moe_forward", load_library().myl_moe_forward(self.ctx.handle, self._h, _p(xs),
                                                                 xs.shape[0], _p(y)))
        return y

    def dev(self, x, out, topk_idx=None, topk_prob=None, stream=None) -> None:
        _check("myl_moe_dev", load_library().myl_moe_dev(
            self.ctx.handle, self._h, _p(x), x.shape[0], x.stride(0), _p(out), out.stride(0),
            _p(topk_idx), _p(topk_prob), _stream_ptr(stream)))

    def route_dev(self, x, topk_idx, topk_prob, stream=None) -> None:
        _check("myl_moe_route_dev", load_library().myl_moe_route_dev(
            self.ctx.handle, self._h, _p(x), x.shape[0], x.stride(0), _p(topk_idx), _p(topk_prob),
            _stream_ptr(stream)))

    def experts_dev(self, x, expert_ids, y, stream=None) -> None:
        _check("myl_moe_experts_dev", load_library().myl_moe_experts_dev(
            self.ctx.handle, self._h, _p(x), x.shape[0], x.stride(0), _p(expert_ids), _p(y),
            y.stride(0), _stream_ptr(stream)))

    def combine_dev(self, y, topk_prob, shared_out, out, stream=None) -> None:
        _check("myl_moe_combine_dev", load_library().myl_moe_combine_dev(
            self.ctx.handle, self._h, _p(y), y.stride(0), _p(topk_prob), _p(shared_out),
            shared_out.stride(0) if shared_out is not None else 0, out.shape[0], _p(out),
            out.stride(0), _stream_ptr(stream)))


def sha256(data: bytes) -> bytes:
    """SHA-256 (FIPS 180-4), the digest the artifact loader checks."""
    out = (C.c_uint8 * 32)()
    buf = C.create_string_buffer(bytes(data), len(data))
    _check("myl_sha256", load_library().myl_sha256(C.cast(buf, C.c_void_p), len(data), out))
    return bytes(out)


class Artifact:
    """A θ_v artifact directory (runtime/src/loader.rs:322-560): weights and
    LUT manifests read and verified on the host; 2-D tensors register as
    weights on a context."""

    def __init__(self, path: str):
        h = C.c_void_p()
        _check("myl_artifact_open", load_library().myl_artifact_open(str(path).encode(), C.byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            load_library().myl_artifact_close(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        return int(load_library().myl_artifact_count(self._h))

    def index(self, name: str) -> int:
        i = C.c_int64()
        _check("myl_artifact_find", load_library().myl_artifact_find(self._h, name.encode(), C.byref(i)))
        return i.value

    def tensor(self, name_or_index):
        """(key, original_name, data ndarray int8/int16 of the manifest shape, shifts uint8)."""
        i = name_or_index if isinstance(name_or_index, int) else self.index(name_or_index)
        key, orig = C.c_char_p(), C.c_char_p()
        dtype, ndim = C.c_int(), C.c_int()
        shape = (C.c_int64 * 4)()
        data, shifts = C.c_void_p(), C.c_void_p()
        _check("myl_artifact_tensor", load_library().myl_artifact_tensor(
            self._h, i, C.byref(key), C.byref(orig), C.byref(dtype), C.byref(ndim), shape,
            C.byref(data), C.byref(shifts)))
        shp = tuple(shape[j] for j in range(ndim.value))
        n = int(np.prod(shp)) if shp else 0
        ctype = C.c_int8 if dtype.value == 1 else C.c_int16
        arr = np.ctypeslib.as_array((ctype * max(n, 1)).from_address(data.value or 0))[:n] if n else \
            np.zeros(0, np.int8 if dtype.value == 1 else np.int16)
        rows = shp[0] if shp else 0
        sh = np.ctypeslib.as_array((C.c_uint8 * max(rows, 1)).from_address(shifts.value))[:rows] \
            if rows and shifts.value else np.zeros(0, np.uint8)
        return key.value.decode(), orig.value.decode(), arr.reshape(shp).copy(), sh.copy()

    def register(self, ctx: "Context", name_or_index) -> "Weight":
        """The tensor as a device weight (int16: LM head path A)."""
        i = name_or_index if isinstance(name_or_index, int) else self.index(name_or_index)
        _, _, arr, sh = self.tensor(i)
        h = C.c_void_p()
        _check("myl_artifact_register", load_library().myl_artifact_register(
            ctx.handle, self._h, i, C.byref(h)))
        w = Weight16.__new__(Weight16) if arr.dtype == np.int16 else Weight.__new__(Weight)
        w.ctx, w._h, w.out_features, w.in_features, w.w_shifts = ctx, h, arr.shape[0], arr.shape[1], sh
        return w

    def lut(self, name: str) -> np.ndarray:
        data, n = C.c_void_p(), C.c_int64()
        _check("myl_artifact_lut", load_library().myl_artifact_lut(self._h, name.encode(), C.byref(data),
                                                                     C.byref(n)))
        if n.value == 0:
            return np.zeros(0, np.int16)
        return np.ctypeslib.as_array((C.c_int16 * n.value).from_address(data.value)).copy()


IPC_HANDLE_BYTES = 64
WIRE_HEADER_BYTES = 84
WIRE_FLAG_STARTS_GENERATION = 0x1
WIRE_FLAG_ABORT = 0x2
WIRE_FLAG_TOKEN_INPUT = 0x4
_WIRE_FIELDS = ("version", "theta_v_hash", "request_id", "sequence_id", "stage_id",
                "token_position", "payload_len", "flags", "reserved")


class WireMeta(C.Structure):
    """myl_wire_meta: the header fields of a pipeline frame (codec.rs:15-29)."""

    _fields_ = [(f, C.c_uint64) for f in _WIRE_FIELDS] + [("crc", C.c_uint32)]

    def as_dict(self) -> dict:
        return {f: getattr(self, f) for f in _WIRE_FIELDS + ("crc",)}

    @classmethod
    def from_dict(cls, d: dict) -> "WireMeta":
        m = cls()
        for f in _WIRE_FIELDS + ("crc",):
            setattr(m, f, int(d.get(f, 0)))
        return m


def crc32(data) -> int:
    """CRC-32 of bytes (host)."""
    b = np.frombuffer(bytes(data), np.uint8)
    return int(load_library().myl_crc32(_p(b) if b.size else None, b.size))


def wire_encode(meta: dict, values) -> bytes:
    """encode_message (codec.rs:86-111): the frame of int16 values."""
    v = _c(np.asarray(values).reshape(-1), np.int16)
    out = np.zeros(load_library().myl_wire_frame_bytes(v.size), np.uint8)
    ln = C.c_uint64()
    m = WireMeta.from_dict(meta)
    _check("myl_wire_encode", load_library().myl_wire_encode(
        C.byref(m), _p(v) if v.size else None, v.size, _p(out), out.size, C.byref(ln)))
    return out[: ln.value].tobytes()


def wire_decode(frame: bytes) -> tuple[dict, np.ndarray]:
    """decode_message (codec.rs:113-178): (meta, int16 values); malformed
    frames raise MylError with MYL_ERR_CORRUPT."""
    buf = np.frombuffer(bytes(frame), np.uint8)
    m = WireMeta()
    n = C.c_uint64()
    L = load_library()
    _check("myl_wire_decode", L.myl_wire_decode(_p(buf) if buf.size else None, buf.size,
                                                C.byref(m), None, 0, C.byref(n)))
    v = np.zeros(n.value, np.int16)
    _check("myl_wire_decode", L.myl_wire_decode(_p(buf), buf.size, C.byref(m),
                                                _p(v) if v.size else None, v.size, C.byref(n)))
    return m.as_dict(), v


def pack_tokens(tokens) -> np.ndarray:
    """Token ids as int16 payload values (codec.rs:38-47)."""
    t = _c(np.asarray(tokens, dtype=np.uint64).astype(np.uint32), np.uint32)
    out = np.zeros(2 * t.size, np.int16)
    _check("myl_wire_pack_tokens", load_library().myl_wire_pack_tokens(
        _p(t) if t.size else None, t.size, _p(out) if out.size else None))
    return out


def unpack_tokens(values) -> np.ndarray:
    """Inverse of pack_tokens (codec.rs:49-63); an odd count raises."""
    v = _c(np.asarray(values).reshape(-1), np.int16)
    out = np.zeros(v.size // 2, np.uint32)
    _check("myl_wire_unpack_tokens", load_library().myl_wire_unpack_tokens(
        _p(v) if v.size else None, v.size, _p(out) if out.size else None))
    return out


def selection_key(logit: int, index: int) -> int:
    """The key myl_argmax_keys_dev gives logit at vocab index: larger logit
    first, then the lower index (argmax_int, sampling.rs:8-18)."""
    return int(logit) * (1 << 32) + (0xFFFFFFFF - int(index))


def keys_to_tokens(keys):
    """(token ids, winning logits) of selection keys (numpy or torch int64)."""
    low = keys & 0xFFFFFFFF
    return 0xFFFFFFFF - low, keys >> 32


def _stream_ptr(stream) -> int | None:
    if stream is None:
        try:
            import torch
            return int(torch.cuda.current_stream().cuda_stream) or None
        except Exception:
            return None
    if hasattr(stream, "cuda_stream"):
        return int(stream.cuda_stream) or None
    return int(stream) or None


# ---- the reference's free functions ---------------------------------------------

_default_ctx: Context | None = None
_cache: dict = {}


def default_context() -> Context:
    global _default_ctx
    if _default_ctx is None:
        _default_ctx = Context(0)
    return _default_ctx


def _cached_weight(W, in_features: int, w_shifts) -> Weight:
    W = np.asarray(W, dtype=np.int8)
    w_shifts = _c(w_shifts, np.uint8)
    if in_features <= 0 or W.size != in_features * w_shifts.size:
        # linear.rs:51-58: "{} Gewichte passen nicht zu {} Zeilen à {} Elementen"
        raise MylError("linear_w8a16", MYL_ERR_SHAPE,
                       f"{W.size} weights do not fit {w_shifts.size} rows of {in_features} elements")
    key = (W.__array_interface__["data"][0], W.size, in_features, w_shifts.tobytes())
    w = _cache.get(key)
    if w is None:
        w = Weight(default_context(), W.reshape(-1), in_features, w_shifts)
        _cache[key] = w
    return w


def clear_weight_cache() -> None:
    _cache.clear()
    _mlp_cache.clear()


def linear_w8a16(x, W, in_features: int, w_shifts, act_frac_bits: int, out_frac_bits: int) -> np.ndarray:
    """kernels/src/linear.rs:43 on the B200 (x: [K] or [M, K])."""
    return _cached_weight(W, in_features, w_shifts).linear(x, act_frac_bits, int(out_frac_bits))


def linear_w8a16_pc(x, W, in_features: int, w_shifts, act_frac_bits: int, out_frac_bits) -> np.ndarray:
    """kernels/src/linear.rs:87 (one out_frac per output channel)."""
    of = _c(out_frac_bits, np.uint8)
    if of.size != np.asarray(w_shifts).size:
        raise MylError("linear_w8a16_pc", MYL_ERR_SHAPE, "one out_frac per channel (Fund 20)")
    return _cached_weight(W, in_features, w_shifts).linear(x, act_frac_bits, of)


def add_bias_linear_w8a16(x, W, in_features: int, w_shifts, act_frac_bits: int, out_frac_bits: int,
                          bias, bias_shifts) -> np.ndarray:
    """linear_w8a16 followed by add_bias_i16 (linear.rs:43, :132), as q/k/v use it."""
    return _cached_weight(W, in_features, w_shifts).linear_bias(x, act_frac_bits, int(out_frac_bits),
                                                                bias, bias_shifts)


_mlp_cache: dict = {}


def mlp_int(x, W_gate, W_up, W_down, hidden_size: int, intermediate_size: int, gate_w_shifts,
            up_w_shifts, down_w_shifts, silu_lut, in_frac_bits: int, gate_out_frac: int,
            up_out_frac: int, down_in_frac: int, silu_in_frac: int, silu_lut_offset: int,
            silu_out_frac: int, out_frac_bits) -> np.ndarray:
    """kernels/src/mlp.rs:28 on the B200 (x: [hidden] or [M, hidden])."""
    arrs = [np.asarray(a) for a in (W_gate, W_up, W_down, gate_w_shifts, up_w_shifts, down_w_shifts,
                                    silu_lut, out_frac_bits)]
    key = tuple((a.__array_interface__["data"][0], a.size, a.dtype.str) for a in arrs) + (
        hidden_size, intermediate_size, in_frac_bits, gate_out_frac, up_out_frac, down_in_frac,
        silu_in_frac, silu_lut_offset, silu_out_frac,
        np.asarray(gate_w_shifts).tobytes(), np.asarray(up_w_shifts).tobytes(),
        np.asarray(down_w_shifts).tobytes(), np.asarray(out_frac_bits).tobytes())
    m = _mlp_cache.get(key)
    if m is None:
        m = Mlp(default_context(), W_gate, W_up, W_down, hidden_size, intermediate_size, gate_w_shifts,
                up_w_shifts, down_w_shifts, silu_lut, in_frac_bits, gate_out_frac, up_out_frac,
                down_in_frac, silu_in_frac, silu_lut_offset, silu_out_frac, out_frac_bits)
        _mlp_cache[key] = m
    return m(x)


def lm_head_w8a16_i32(x, W, in_features: int, w_shifts, final_norm_frac: int, logit_frac: int) -> np.ndarray:
    """runtime/src/model.rs:297-307: logits clamped to i32."""
    return _cached_weight(W, in_features, w_shifts).lm_head(x, final_norm_frac, logit_frac)


class CudaBackend:
    """The reference's Backend trait slot for CUDA (kernels/src/backends/cuda.rs),
    with a real computing path for linear_w8a16 (backend.rs:39-49)."""

    def __init__(self, device_id: int = 0):
        self._ctx = Context(device_id)

    @classmethod
    def init(cls, device_id: int = 0) -> "CudaBackend":
        return cls(device_id)

    def name(self) -> str:
        return "cuda"

    def hardware_family(self) -> str:
        return "nvidia-gpu"

    def feature_tag(self) -> str:
        return "cuda-sm100a"

    def device_id(self) -> int:
        return self._ctx.device

    def sm_version(self) -> int:
        return self._ctx.sm_version

    def linear_w8a16(self, x, W, out, in_features: int, out_features: int, w_shifts,
                     act_frac: int, out_frac: int) -> None:
        x = _c(x, np.int16)
        W = np.ascontiguousarray(np.asarray(W, dtype=np.int8))
        w_shifts = _c(w_shifts, np.uint8)
        if not (isinstance(out, np.ndarray) and out.dtype == np.int16 and out.flags.c_contiguous):
            raise MylError("linear_w8a16", MYL_ERR_ARG, "out must be a contiguous int16 numpy array")
        if (W.size != in_features * out_features or w_shifts.size < out_features
                or out.size < out_features or x.size < in_features):
            raise MylError("linear_w8a16", MYL_ERR_SHAPE, "argument lengths do not match the shape")
        _check("myl_backend_linear_w8a16", load_library().myl_backend_linear_w8a16(
            self._ctx.handle, _p(x), _p(W), _p(out), in_features, out_features, _p(w_shifts),
            act_frac, out_frac))

    def mlp(self, x, W_gate, W_up, W_down, out, gate_w_shifts, up_w_shifts, down_w_shifts, silu_lut,
            in_frac: int, gate_out_frac: int, up_out_frac: int, down_in_frac: int, silu_in_frac: int,
            silu_lut_offset: int, silu_out_frac: int, out_frac) -> None:
        """Backend::mlp (kernels/src/backend.rs:107-126): hidden = x.len(),
        intermediate = W_gate.len() / hidden; writes into out."""
        x = _c(x, np.int16)
        hidden = x.size
        inter = np.asarray(W_gate).size // max(hidden, 1)
        y = mlp_int(x, W_gate, W_up, W_down, hidden, inter, gate_w_shifts, up_w_shifts, down_w_shifts,
                    silu_lut, in_frac, gate_out_frac, up_out_frac, down_in_frac, silu_in_frac,
                    silu_lut_offset, silu_out_frac, out_frac)
        out[:hidden] = y
