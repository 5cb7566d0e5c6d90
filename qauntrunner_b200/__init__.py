"""qauntrunner_b200 -- B200 (sm_100a) MoE FFN layer for QuantRunner.

Python view of the C ABI in include/qrmoe.h (libqrmoe.so, built in-tree by
qauntrunner_b200.build).  It mirrors what the reference's StreamingEngine does
with one MoE layer (src/QuantRunner.Core/Runtime/StreamingEngine.cs:626-790):
a layer is described by the ModelConfig MoE fields, its tensors are uploaded
under their canonical roles (ffn_norm, router, router_bias, e{j}.w_gate/w_up/
w_down, sw_*), and forward() runs RMSNorm -> router -> top-k -> experts ->
combine for a batch of tokens.  There is no CPU fallback: every call goes to
the CUDA library and fails loudly without it.
"""
import ctypes as C
import enum
import os

import numpy as np

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "lib", "libqrmoe.so")
_ROOT = os.path.dirname(_PKG)
HEADER_PATH = os.path.join(_ROOT, "include", "qrmoe.h")


class QuantFormat(enum.IntEnum):
    """QuantFormat ids of the .qw format (src/QuantRunner.Core/Dtypes.cs:6-26)."""
    F32 = 0
    F16 = 1
    BF16 = 2
    Q4_0 = 3
    Q8_0 = 4
    Q2_K = 5
    Q4_K = 6
    Q6_K = 7
    TRI = 8
    I8_BLK = 9
    Q3_K = 10
    Q5_K = 11
    B1 = 12
    B1X = 13
    T1E = 14
    T1E_LO = 15


TRI_LEGACY = 108  # quantiser selector for BlockQuantizer.QuantizeTriLegacy (same storage as TRI)
BLOCK_SPEC = {0: (1, 4), 1: (1, 2), 2: (1, 2), 3: (32, 20), 4: (32, 34), 5: (256, 84), 6: (256, 144), 7: (256, 210),
              8: (64, 18), 9: (256, 258), 10: (256, 110), 11: (256, 176), 12: (256, 34), 13: (256, 47), 14: (256, 40),
              15: (256, 32)}
GATE, UP, DOWN = 0, 1, 2
SHARED_EXPERT = -1
APPLY_NORM, ADD_RESIDUAL = 1, 2
STAGES = ("route", "topk", "dispatch", "gateup", "down", "combine")
STAGE_COUNT = len(STAGES)
EP_STAGES = ("route", "records", "gateup", "down", "outputs", "combine")
E_INVALID, E_FORMAT, E_SIZE, E_STATE, E_CUDA, E_NCCL, E_TIMEOUT, E_NOMEM, E_CAPACITY = range(-1, -10, -1)
ERRORS = {-1: "QRM_E_INVALID", -2: "QRM_E_FORMAT", -3: "QRM_E_SIZE", -4: "QRM_E_STATE", -5: "QRM_E_CUDA",
          -6: "QRM_E_NCCL", -7: "QRM_E_TIMEOUT", -8: "QRM_E_NOMEM", -9: "QRM_E_CAPACITY"}


NCCL_ID_BYTES = 128


def nccl_unique_id():
    """A new NCCL unique id (128 bytes) for qrm_create_ep; made on one rank and
    passed to all of them by the host."""
    buf = C.create_string_buffer(NCCL_ID_BYTES)
    _check(lib().qrm_nccl_unique_id(buf))
    return buf.raw


class QrmError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


def tensor_bytes(n, fmt):
    """Dtypes.TensorBytes (Dtypes.cs:60-65)."""
    bs, bb = BLOCK_SPEC[int(QuantFormat.TRI if fmt == TRI_LEGACY else fmt)]
    if n % bs:
        raise ValueError(f"element count {n} not a multiple of block size {bs}")
    return n // bs * bb


class LayerDesc(C.Structure):
    _fields_ = [("d_model", C.c_int32), ("n_experts", C.c_int32), ("n_active", C.c_int32),
                ("expert_ffn", C.c_int32), ("moe_sigmoid", C.c_int32), ("routed_scale", C.c_float),
                ("n_shared", C.c_int32), ("swiglu_limit", C.c_float), ("rms_eps", C.c_float),
                ("fmt_gate", C.c_int32), ("fmt_up", C.c_int32), ("fmt_down", C.c_int32),
                ("fmt_sh_gate", C.c_int32), ("fmt_sh_up", C.c_int32), ("fmt_sh_down", C.c_int32),
                ("device", C.c_int32), ("max_tokens", C.c_int32)]


P = C.c_void_p
_SIGS = {
    "qrm_version": (C.c_int, []),
    "qrm_last_error": (C.c_char_p, []),
    "qrm_create": (C.c_int, [C.POINTER(LayerDesc), C.POINTER(P)]),
    "qrm_destroy": (None, [P]),
    "qrm_layer_get_desc": (C.c_int, [P, C.POINTER(LayerDesc)]),
    "qrm_qw_layer_desc": (C.c_int, [C.c_char_p, C.c_int, C.c_int, C.c_int, C.POINTER(LayerDesc)]),
    "qrm_load_qw": (C.c_int, [P, C.c_char_p, C.c_int]),
    "qrm_upload_norm": (C.c_int, [P, P]),
    "qrm_upload_router": (C.c_int, [P, P, P]),
    "qrm_upload_logit_offset": (C.c_int, [P, P]),
    "qrm_upload_expert": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P, C.c_size_t]),
    "qrm_upload_expert_device": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P, C.c_size_t]),
    "qrm_download_expert": (C.c_int, [P, C.c_int, C.c_int, P, C.c_size_t]),
    "qrm_forward": (C.c_int, [P, P, C.c_int, C.c_int, P, P, P]),
    "qrm_forward_device": (C.c_int, [P, P, C.c_int, C.c_int, P, P, P, P]),
    "qrm_sync": (C.c_int, [P]),
    "qrm_last_dispatch": (C.c_int, [P, P, P]),
    "qrm_last_router": (C.c_int, [P, P, P]),
    "qrm_set_profiling": (C.c_int, [P, C.c_int]),
    "qrm_last_profile": (C.c_int, [P, P, P]),
    "qrm_last_launch_count": (C.c_int, [P, P]),
    "qrm_matrix_create": (C.c_int, [C.c_int, C.c_int, C.c_int64, C.c_int64, P, C.c_size_t, C.POINTER(P)]),
    "qrm_matrix_destroy": (None, [P]),
    "qrm_matrix_gemv": (C.c_int, [P, P, C.c_int, P, P]),
    "qrm_matrix_gemv_static": (C.c_int, [P, P, C.c_int, P, P]),
    "qrm_stack_create": (C.c_int, [C.POINTER(LayerDesc), C.c_int, C.c_size_t, C.POINTER(P)]),
    "qrm_stack_destroy": (None, [P]),
    "qrm_stack_layer": (C.c_int, [P, C.c_int, C.POINTER(P)]),
    "qrm_stack_info": (C.c_int, [P, P, P]),
    "qrm_stack_load_qw": (C.c_int, [P, C.c_char_p, C.c_int]),
    "qrm_stack_forward_device": (C.c_int, [P, P, C.c_int, C.c_int, P, P]),
    "qrm_stack_sync": (C.c_int, [P]),
    "qrm_ffn_create": (C.c_int, [P, P, P, C.c_int, C.POINTER(P)]),
    "qrm_ffn_destroy": (None, [P]),
    "qrm_ffn_forward": (C.c_int, [P, P, P, C.c_int, C.c_float, P, P]),
    "qrm_nccl_unique_id": (C.c_int, [P]),
    "qrm_create_ep": (C.c_int, [C.POINTER(LayerDesc), C.c_int, C.c_int, P, C.POINTER(P)]),
    "qrm_expert_range": (C.c_int, [P, P, P]),
    "qrm_ep_transport": (C.c_int, [P, P]),
    "qrm_last_profile_ep": (C.c_int, [P, P]),
    "qrm_selftest_expf": (C.c_int, [C.c_uint32, C.c_uint32, P, P]),
    "qrm_selftest_waits": (C.c_int, [C.c_int, C.c_int64, P]),
    "qrm_synth_gaussian": (C.c_int, [P, C.c_int64, C.c_uint64, C.c_float, P]),
    "qrm_synth_quantize": (C.c_int, [C.c_int, P, C.c_int64, P, P]),
}

_lib = None


def lib():
    """Loads libqrmoe.so (raises if it was not built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing; build it with `python -m qauntrunner_b200.build`")
        # libqrmoe.so resolves libnccl.so.2 at load time: in a process that also
        # uses torch, torch's (newer) NCCL must be the one loaded first
        try:
            import torch  # noqa: F401
        except ImportError:
            pass
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def header_symbols():
    """Function names declared in include/qrmoe.h."""
    import re
    with open(HEADER_PATH) as fh:
        txt = fh.read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(qrm_\w+)\s*\(", txt, re.M)))


def _check(rc):
    if rc != 0:
        raise QrmError(rc, lib().qrm_last_error().decode())
    return rc


def _ptr(a):
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data_as(P).value


def qw_layer_desc(path, layer_index, device=0, max_tokens=1):
    """LayerDesc of MoE layer `layer_index` of a .qw file, from its header
    (qrm_qw_layer_desc; no GPU work)."""
    d = LayerDesc()
    _check(lib().qrm_qw_layer_desc(os.fsencode(path), layer_index, device, max_tokens, C.byref(d)))
    return d


class MoeLayer:
    """One MoE FFN layer resident on a GPU.

    Arguments mirror ModelConfig (src/QuantRunner.Core/Models/ModelConfig.cs):
    dim, n_experts, n_active, expert_ffn, moe_sigmoid, routed_scale,
    n_shared, swiglu_limit, rms_eps; plus the storage formats of the routed
    and shared expert matrices, the device and the largest token batch.
    """

    def __init__(self, d_model, n_experts, n_active, expert_ffn, moe_sigmoid=False, routed_scale=1.0,
                 n_shared=0, swiglu_limit=0.0, rms_eps=1e-5, fmt=(6, 6, 6), shared_fmt=None, device=0,
                 max_tokens=1, rank=0, world=1, nccl_id=None):
        """rank / world / nccl_id (bytes from nccl_unique_id() on one rank): an
        expert-parallel layer holding the routed experts of expert_range()."""
        shared_fmt = shared_fmt or fmt
        self.desc = LayerDesc(d_model, n_experts, n_active, expert_ffn, int(bool(moe_sigmoid)), routed_scale,
                              n_shared, swiglu_limit, rms_eps, int(fmt[0]), int(fmt[1]), int(fmt[2]),
                              int(shared_fmt[0]), int(shared_fmt[1]), int(shared_fmt[2]), device, max_tokens)
        self.k = min(n_active, 8)
        self.rank, self.world = rank, world
        h = P()
        if world > 1:
            if nccl_id is None or len(nccl_id) != NCCL_ID_BYTES:
                raise ValueError("an expert-parallel layer needs the 128-byte NCCL id of nccl_unique_id()")
            buf = C.create_string_buffer(bytes(nccl_id), NCCL_ID_BYTES)
            _check(lib().qrm_create_ep(C.byref(self.desc), rank, world, buf, C.byref(h)))
        else:
            _check(lib().qrm_create(C.byref(self.desc), C.byref(h)))
        self._h = h

    @classmethod
    def from_qw(cls, path, layer_index, device=0, max_tokens=1, rank=0, world=1, nccl_id=None):
        """MoE layer `layer_index` of a .qw file (ModelStore.Open), its
        description from the file's header and its tensors uploaded by their
        canonical names."""
        d = qw_layer_desc(path, layer_index, device, max_tokens)
        L = cls(d.d_model, d.n_experts, d.n_active, d.expert_ffn, moe_sigmoid=bool(d.moe_sigmoid),
                routed_scale=d.routed_scale, n_shared=d.n_shared, swiglu_limit=d.swiglu_limit, rms_eps=d.rms_eps,
                fmt=(d.fmt_gate, d.fmt_up, d.fmt_down), shared_fmt=(d.fmt_sh_gate, d.fmt_sh_up, d.fmt_sh_down),
                device=device, max_tokens=max_tokens, rank=rank, world=world, nccl_id=nccl_id)
        try:
            _check(lib().qrm_load_qw(L._h, os.fsencode(path), layer_index))
        except Exception:
            L.close()
            raise
        return L

    def get_desc(self):
        """The qrm_layer_desc the library holds for this layer."""
        d = LayerDesc()
        _check(lib().qrm_layer_get_desc(self._h, C.byref(d)))
        return d

    def expert_range(self):
        """(first, count) of the routed experts this layer holds."""
        a, b = C.c_int(0), C.c_int(0)
        _check(lib().qrm_expert_range(self._h, C.byref(a), C.byref(b)))
        return a.value, b.value

    def ep_transport(self):
        """"single", "nccl" or "peer" (NVLink stores into the peers' memory)."""
        v = C.c_int(0)
        _check(lib().qrm_ep_transport(self._h, C.byref(v)))
        return ("single", "nccl", "peer")[v.value]

    def close(self):
        if getattr(self, "_h", None):
            if not getattr(self, "_borrowed", False):   # a stack's layer belongs to the stack
                lib().qrm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    # ---- uploads
    def upload_norm(self, w):
        w = np.ascontiguousarray(w, dtype=np.float32)
        _check(lib().qrm_upload_norm(self._h, _ptr(w)))

    def upload_router(self, w, bias=None):
        w = np.ascontiguousarray(w, dtype=np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        _check(lib().qrm_upload_router(self._h, _ptr(w), _ptr(b)))

    def upload_logit_offset(self, off):
        o = None if off is None else np.ascontiguousarray(off, dtype=np.float32)
        _check(lib().qrm_upload_logit_offset(self._h, _ptr(o)))

    def upload_expert(self, expert, which, fmt, data):
        b = np.ascontiguousarray(data, dtype=np.uint8)
        _check(lib().qrm_upload_expert(self._h, expert, which, int(fmt), _ptr(b), b.nbytes))

    def upload_expert_device(self, expert, which, fmt, dev_ptr, nbytes):
        _check(lib().qrm_upload_expert_device(self._h, expert, which, int(fmt), dev_ptr, nbytes))

    def download_expert(self, expert, which, nbytes):
        out = np.zeros(nbytes, np.uint8)
        _check(lib().qrm_download_expert(self._h, expert, which, _ptr(out), nbytes))
        return out

    # ---- forward
    def forward(self, x, apply_norm=True, add_residual=False):
        """Host arrays in and out (synchronous).  Returns (out, topk_idx, topk_w)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0]
        out = np.empty_like(x)
        idx = np.empty((T, self.k), np.int32)
        w = np.empty((T, self.k), np.float32)
        flags = (APPLY_NORM if apply_norm else 0) | (ADD_RESIDUAL if add_residual else 0)
        _check(lib().qrm_forward(self._h, _ptr(x), T, flags, _ptr(out), _ptr(idx), _ptr(w)))
        return out, idx, w

    def forward_into(self, x, flags, out, idx=None, w=None):
        """qrm_forward on caller-owned host arrays (pageable memory, no
        allocation here): the call the C# shim makes."""
        _check(lib().qrm_forward(self._h, _ptr(x), x.shape[0], flags, _ptr(out), _ptr(idx), _ptr(w)))

    def forward_device(self, x_ptr, T, out_ptr, flags=APPLY_NORM, idx_ptr=None, w_ptr=None, stream=None):
        _check(lib().qrm_forward_device(self._h, x_ptr, T, flags, out_ptr, idx_ptr, w_ptr, stream))

    def sync(self):
        _check(lib().qrm_sync(self._h))

    def last_dispatch(self, T):
        perm = np.zeros(T * self.k, np.int32)
        off = np.zeros(self.desc.n_experts + 1, np.int32)
        _check(lib().qrm_last_dispatch(self._h, _ptr(perm), _ptr(off)))
        return perm, off

    def set_profiling(self, on=True):
        _check(lib().qrm_set_profiling(self._h, int(bool(on))))

    def last_profile(self):
        """(ms per stage, algorithmic bytes per stage) of the last forward; stages:
        route, topk, dispatch, gate/up, down, combine."""
        ms = np.zeros(STAGE_COUNT, np.float32)
        by = np.zeros(STAGE_COUNT, np.float64)
        _check(lib().qrm_last_profile(self._h, _ptr(ms), _ptr(by)))
        return ms, by

    def last_profile_ep(self):
        """ms per stage of the last expert-parallel forward; stages: route,
        records, gate/up, down, outputs, combine (EP_STAGES)."""
        ms = np.zeros(len(EP_STAGES), np.float32)
        _check(lib().qrm_last_profile_ep(self._h, _ptr(ms)))
        return ms

    def last_launch_count(self):
        """Kernel launches of this library in the last forward."""
        n = C.c_int(0)
        _check(lib().qrm_last_launch_count(self._h, C.byref(n)))
        return n.value

    def last_router(self, T):
        logits = np.zeros((T, self.desc.n_experts), np.float32)
        xn = np.zeros((T, self.desc.d_model), np.float32)
        _check(lib().qrm_last_router(self._h, _ptr(logits), _ptr(xn)))
        return logits, xn


class Matrix:
    """A [rows x cols] quantised matrix in HBM: DotKernels.MatVecParallel /
    DotKernels.GEMM (src/QuantRunner.Core/Kernels/DotKernels.cs:610-660) on the GPU."""

    def __init__(self, fmt, rows, cols, data, device=0):
        b = np.ascontiguousarray(data, dtype=np.uint8)
        h = P()
        _check(lib().qrm_matrix_create(device, int(fmt), rows, cols, _ptr(b), b.nbytes, C.byref(h)))
        self._h, self.rows, self.cols = h, rows, cols

    def gemv(self, x_ptr, T, y_ptr, stream=None):
        _check(lib().qrm_matrix_gemv(self._h, x_ptr, T, y_ptr, stream))

    def gemv_static(self, x_ptr, T, y_ptr, stream=None):
        """gemv with the activation tables in the library's fixed per-device
        scratch (no allocation; concurrent calls on one device race)."""
        _check(lib().qrm_matrix_gemv_static(self._h, x_ptr, T, y_ptr, stream))

    def close(self):
        if getattr(self, "_h", None):
            lib().qrm_matrix_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MoeStack:
    """n MoE layers of one shape on a device-resident residual stream
    (qrm_stack_*): the first n_resident layers' weights stay in HBM, the rest
    stream from pinned host memory through two device slots when hbm_budget
    (bytes, 0 = no limit) does not hold them all."""

    def __init__(self, n_layers, d_model, n_experts, n_active, expert_ffn, hbm_budget=0, moe_sigmoid=False,
                 routed_scale=1.0, n_shared=0, swiglu_limit=0.0, rms_eps=1e-5, fmt=(6, 6, 6), shared_fmt=None,
                 device=0, max_tokens=1):
        shared_fmt = shared_fmt or fmt
        self.desc = LayerDesc(d_model, n_experts, n_active, expert_ffn, int(bool(moe_sigmoid)), routed_scale,
                              n_shared, swiglu_limit, rms_eps, int(fmt[0]), int(fmt[1]), int(fmt[2]),
                              int(shared_fmt[0]), int(shared_fmt[1]), int(shared_fmt[2]), device, max_tokens)
        h = P()
        _check(lib().qrm_stack_create(C.byref(self.desc), n_layers, int(hbm_budget), C.byref(h)))
        self._h = h
        self.n_layers = n_layers
        self.layers = []
        for i in range(n_layers):
            lh = P()
            _check(lib().qrm_stack_layer(h, i, C.byref(lh)))
            L = MoeLayer.__new__(MoeLayer)
            L._h, L._borrowed, L.desc, L.k, L.rank, L.world = lh, True, self.desc, min(n_active, 8), 0, 1
            self.layers.append(L)

    def info(self):
        """(resident layers, expert bytes of one layer)."""
        a, b = C.c_int(0), C.c_size_t(0)
        _check(lib().qrm_stack_info(self._h, C.byref(a), C.byref(b)))
        return a.value, b.value

    def load_qw(self, path, first_layer=0):
        _check(lib().qrm_stack_load_qw(self._h, os.fsencode(path), first_layer))

    def forward_device(self, x_ptr, T, out_ptr, flags=APPLY_NORM | ADD_RESIDUAL, stream=None):
        _check(lib().qrm_stack_forward_device(self._h, x_ptr, T, flags, out_ptr, stream))

    def sync(self):
        _check(lib().qrm_stack_sync(self._h))

    def close(self):
        for L in getattr(self, "layers", []):
            L._h = None
        if getattr(self, "_h", None):
            lib().qrm_stack_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DenseFfn:
    """StreamingEngine.DenseFfn / DenseFfnOut (StreamingEngine.cs:599-622) on
    the GPU from three Matrix objects (gate, up [f x d]; down [d x f])."""

    def __init__(self, gate, up, down, max_tokens=1):
        h = P()
        _check(lib().qrm_ffn_create(gate._h, up._h, down._h, max_tokens, C.byref(h)))
        self._h = h
        self._mats = (gate, up, down)   # the FFN refers to them: keep them alive

    def forward(self, xn_ptr, x_ptr, T, out_ptr, swiglu_limit=0.0, stream=None):
        """out = x + W_down SwiGLU(W_gate xn, W_up xn) (x_ptr None: without x)."""
        _check(lib().qrm_ffn_forward(self._h, xn_ptr, x_ptr, T, swiglu_limit, out_ptr, stream))

    def close(self):
        if getattr(self, "_h", None):
            lib().qrm_ffn_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def synth_gaussian(dev_ptr, n, seed, sigma, stream=None):
    _check(lib().qrm_synth_gaussian(dev_ptr, n, seed, sigma, stream))


def synth_quantize(fmt, src_ptr, n, dst_ptr, stream=None):
    _check(lib().qrm_synth_quantize(int(fmt), src_ptr, n, dst_ptr, stream))
