"""Loads libmq.so (built in-tree next to this file) and declares its C ABI (include/mq.h)."""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
library_path = os.path.join(_HERE, "libmq.so")

c_int, c_i64, c_vp, c_char_p, c_size = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t

# name -> (restype, argtypes), in include/mq.h order.
SIGNATURES = {
    "mq_last_error": (c_char_p, []),
    "mq_version": (c_int, []),
    "mq_device_status": (c_int, [c_int, c_vp]),
    "mq_unpack_q4": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_int, c_vp]),
    "mq_gemv_q4": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp, c_i64, c_i64, c_int, c_int, c_int, c_vp]),
    "mq_gemm_q4_workspace_size": (c_size, [c_i64, c_i64, c_int]),
    "mq_gemm_q4": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp, c_i64, c_i64, c_i64, c_int, c_int, c_vp, c_size, c_vp]),
    "mq_gemm_q4_noalloc": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_int, c_int, c_vp]),
    "mq_tgemv": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_int, c_vp]),
    "mq_tgemv_head": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_int, c_vp]),
    "mq_head_argmax": (c_int, [c_vp, c_i64, c_int, c_vp, c_vp]),
    "mq_gate_up_q4": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp, c_i64, c_i64, c_int, c_int, c_vp]),
    "mq_moe_gate_up_q4": (c_int, [c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_int, c_vp]),
    "mq_gemm_t2": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_int, c_vp, c_size, c_vp]),
    "mq_moe_router": (c_int, [c_vp, c_vp, c_vp, c_i64, c_int, c_i64, c_vp]),
    "mq_moe_route": (c_int, [c_vp, c_vp, c_vp, c_i64, c_int, c_int, c_vp]),
    "mq_moe_group": (c_int, [c_vp, c_i64, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "mq_moe_route_group": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_int, c_int, c_i64, c_int, c_vp, c_vp, c_vp,
                                   c_vp, c_vp, c_vp, c_vp]),
    "mq_moe_layer": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_int, c_int, c_i64,
                             c_i64, c_int, c_int, c_vp, c_size, c_vp]),
    "mq_ep_plan": (c_int, [c_vp, c_i64, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "mq_moe_gather": (c_int, [c_vp, c_int, c_vp, c_i64, c_int, c_i64, c_vp, c_vp]),
    "mq_moe_gemm_q4": (c_int, [c_int, c_vp, c_vp, c_vp, c_i64, c_i64, c_int, c_i64, c_int, c_vp, c_vp, c_int, c_int,
                               c_vp, c_vp]),
    "mq_moe_gemv_q4": (c_int, [c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_i64, c_int, c_int, c_vp]),
    "mq_moe_silu_mul": (c_int, [c_vp, c_vp, c_i64, c_i64, c_vp]),
    "mq_moe_combine": (c_int, [c_vp, c_vp, c_vp, c_i64, c_int, c_i64, c_int, c_vp, c_vp]),
    "mq_moe_workspace_size": (c_size, [c_i64, c_int, c_int, c_i64, c_i64]),
    "mq_moe_forward": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_int, c_int, c_i64, c_i64,
                               c_int, c_int, c_vp, c_size, c_vp]),
    "mq_quantize_q4": (c_int, [c_vp, c_int, c_i64, c_i64, c_int, c_int, c_vp, c_vp, c_vp]),
    "mq_q4_0_to_words": (c_int, [c_vp, c_i64, c_vp, c_vp, c_vp]),
    "mq_pack_ternary": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp]),
    "mq_ipc_handle": (c_int, [c_vp, c_vp, ctypes.POINTER(c_i64)]),
    "mq_ipc_open": (c_int, [c_vp, c_i64, ctypes.POINTER(c_vp)]),
    "mq_ipc_close": (c_int, [c_vp, c_i64]),
    "mq_ep_dispatch": (c_int, [c_vp, c_int, c_vp, c_vp, c_i64, c_int, c_i64, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp,
                               c_vp, c_vp]),
    "mq_ep_wait": (c_int, [c_vp, c_int, c_int, c_vp, c_vp]),
    "mq_ep_return": (c_int, [c_vp, c_vp, c_vp, c_i64, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "mq_ep_workspace_size": (c_size, [c_i64, c_int, c_i64, c_i64]),
    "mq_ep_expert_step": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_int, c_i64, c_i64, c_int, c_int, c_int,
                                  c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_size, c_vp]),
    "mq_ep_combine": (c_int, [c_vp, c_vp, c_vp, c_i64, c_int, c_i64, c_int, c_vp, c_vp, c_int, c_vp, c_vp]),
    "mq_read_file_to_device": (c_int, [c_vp, c_i64, c_char_p, c_i64, c_vp]),
    "mq_pack_half": (c_int, [c_vp, c_vp, c_i64, c_vp]),
}


class MQError(RuntimeError):
    """A libmq entry point returned a non-zero status (the message is mq_last_error())."""

    def __init__(self, code, message):
        super().__init__(f"{message} (status {code})")
        self.code = code


class _Lib:
    def __init__(self):
        self._dll = None
        self._fns = {}

    def load(self):
        if self._dll is None:
            if not os.path.exists(library_path):
                raise MQError(-3, f"libmq.so is not built ({library_path}); run python mojo-adreno_b200/build.py")
            dll = ctypes.CDLL(library_path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(dll, name)
                fn.restype, fn.argtypes = res, args
            self._dll = dll
        return self._dll

    def __getattr__(self, name):
        return getattr(self.load(), name)

    def call(self, name, *args):
        """Calls entry point `name`; raises MQError on a negative status."""
        fn = self._fns.get(name)
        if fn is None:
            fn = self._fns[name] = getattr(self.load(), name)
        rc = fn(*args)
        if rc < 0:
            raise MQError(rc, f"{name}: {self.load().mq_last_error().decode()}")
        return rc


lib = _Lib()
