"""ctypes binding of ``libb200k.so`` (include/b200k.h).

This is the thin C-ABI shim the front end dispatches through: no PyTorch, no
CPU fallback.  If the library is missing the import of :func:`library` fails
loudly -- a recognised kernel never silently runs anywhere but the GPU.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().parent / "libb200k.so"

B2K_OK, B2K_EINVAL, B2K_EUNSUPPORTED, B2K_ECUDA, B2K_ETIMEOUT, B2K_ESCRATCH = 0, 1, 2, -1, -2, 3
B2K_ENCCL = -3
NOALLOC_SCRATCH_BYTES = 32 << 20
MGPU_ID_BYTES = 128
STATUS_NAMES = {B2K_EINVAL: "EINVAL", B2K_EUNSUPPORTED: "EUNSUPPORTED", B2K_ECUDA: "ECUDA",
                B2K_ETIMEOUT: "ETIMEOUT", B2K_ESCRATCH: "ESCRATCH", B2K_ENCCL: "ENCCL"}

PW_MAX_INPUTS, PW_MAX_INSNS = 8, 48
B_KN, B_NK, A_KM = 0, 1, 2   # A_KM is a flag or-ed into b_layout: A stored [k, m]
K_SD, K_DS = 0, 1

OPCODES = {
    "const": 0, "copy": 1, "add": 2, "subtract": 3, "multiply": 4, "divide": 5, "maximum": 6,
    "minimum": 7, "negative": 8, "reciprocal": 9, "sqrt": 10, "rsqrt": 11, "exp": 12, "relu": 13,
    "abs": 14, "fma": 15, "greater": 16, "greater_equal": 17, "less": 18, "less_equal": 19,
    "where": 20, "log": 21,
}


class B2KError(RuntimeError):
    """A non-OK status from the C ABI, with the library's reason string."""

    def __init__(self, status: int, reason: str, call: str):
        self.status = status
        super().__init__(f"{call}: {STATUS_NAMES.get(status, status)}: {reason}")


class RowParams(C.Structure):
    _fields_ = [("op", C.c_int32), ("sum_div", C.c_float), ("sum_div_ptr", C.c_void_p), ("ms_div", C.c_float),
                ("ms_div_ptr", C.c_void_p), ("eps", C.c_float), ("eps_ptr", C.c_void_p), ("w", C.c_void_p)]


ROW_SUM, ROW_RMSNORM, ROW_L2NORM, ROW_MAX, ROW_MIN, ROW_PROD = 0, 1, 2, 3, 4, 5


(KIND_POINTWISE, KIND_ROW_SOFTMAX, KIND_ROW_OP, KIND_GEMM, KIND_ATTENTION, KIND_AXIS_REDUCE,
 KIND_GEMM_BATCHED) = 1, 2, 3, 4, 5, 6, 7
MAX_ROLES, NO_ARG, ROLE_PW_OUT = 12, -1, 8


class KernelDesc(C.Structure):
    """b2k_kernel_desc: which kernel runs and which positional arguments feed it."""
    _fields_ = [("kind", C.c_int32), ("role", C.c_int32 * MAX_ROLES), ("dims", C.c_int64 * 6),
                ("flags", C.c_int32 * 4), ("values", C.c_float * 4), ("program", C.c_void_p)]


def make_desc(kind: int, roles: dict, dims=(), flags=(), values=(), program=None) -> KernelDesc:
    """Descriptor with `roles` = {role: positional argument index}; unset roles are NO_ARG."""
    desc = KernelDesc()
    desc.kind = kind
    for r in range(MAX_ROLES):
        desc.role[r] = NO_ARG
    for r, idx in roles.items():
        desc.role[r] = idx
    for i, v in enumerate(dims):
        desc.dims[i] = int(v)
    for i, v in enumerate(flags):
        desc.flags[i] = int(v)
    for i, v in enumerate(values):
        desc.values[i] = float(v)
    desc.program = C.cast(C.pointer(program), C.c_void_p) if program is not None else None
    desc._program_ref = program  # keeps the program alive as long as the descriptor
    return desc


class PwInsn(C.Structure):
    _fields_ = [("op", C.c_int32), ("a", C.c_int32), ("b", C.c_int32), ("c", C.c_int32), ("imm", C.c_float)]


class PwProgram(C.Structure):
    _fields_ = [("n_inputs", C.c_int32), ("n_insns", C.c_int32), ("result", C.c_int32),
                ("broadcast", C.c_int32 * PW_MAX_INPUTS), ("offset", C.c_int32 * PW_MAX_INPUTS),
                ("insns", PwInsn * PW_MAX_INSNS)]


class GemmPlan(C.Structure):
    """b2k_gemm_plan_info: the kernel path of one b2k_gemm_tf32x3 call."""
    _fields_ = [("split_mode", C.c_int32), ("tile_width", C.c_int32), ("chunk_split", C.c_int32),
                ("chunks", C.c_int32)]


_P, _I32, _I64, _SZ, _F = C.c_void_p, C.c_int32, C.c_int64, C.c_size_t, C.c_float

# name -> (argtypes without the leading context pointer, or None for no ctx)
SIGNATURES: dict[str, tuple] = {
    "b2k_version": ([], C.c_int),
    "b2k_init": ([C.c_int, C.POINTER(_P)], C.c_int),
    "b2k_destroy": ([_P], C.c_int),
    "b2k_last_error": ([_P], C.c_char_p),
    "b2k_sm_count": ([_P], C.c_int),
    "b2k_malloc": ([_P, C.POINTER(_P), _SZ], C.c_int),
    "b2k_free": ([_P, _P], C.c_int),
    "b2k_memcpy_htod": ([_P, _P, _P, _SZ, _P], C.c_int),
    "b2k_memcpy_dtoh": ([_P, _P, _P, _SZ, _P], C.c_int),
    "b2k_memset": ([_P, _P, C.c_int, _SZ, _P], C.c_int),
    "b2k_host_alloc": ([_P, C.POINTER(_P), _SZ], C.c_int),
    "b2k_host_free": ([_P, _P], C.c_int),
    "b2k_stream_sync": ([_P, _P], C.c_int),
    "b2k_pointwise_f32": ([_P, C.POINTER(PwProgram), C.POINTER(_P), _P, _I64, _P], C.c_int),
    "b2k_row_softmax_f32": ([_P, _P, _P, _I64, _I64, _I64, _I64, _P], C.c_int),
    "b2k_selective_exp_f32": ([_P, _P, _P, _I64, _P], C.c_int),
    "b2k_row_op_f32": ([_P, C.POINTER(RowParams), _P, _P, _I64, _I64, _I64, _I64, _P], C.c_int),
    "b2k_gemm_tf32x3": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _P, _I32, _P], C.c_int),
    "b2k_gemm_tf32x3_scaled": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _P, _I32, _P, C.c_float,
                                _P], C.c_int),
    "b2k_axis_reduce_f32": ([_P, _I32, _P, _P, _I64, _I64, _I64, C.c_float, _P, _P], C.c_int),
    "b2k_gemm_tf32x3_batched": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I32,
                                 _P, _I32, _P], C.c_int),
    "b2k_gemm_set_variant": ([C.c_int], C.c_int),
    "b2k_gemm_set_fused_split": ([C.c_int], C.c_int),
    "b2k_attention_set_fused": ([C.c_int], C.c_int),
    "b2k_attention_tf32x3": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _P, _I32, _P], C.c_int),
    "b2k_gemm_tf32x3_noalloc": ([_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _P, _I32, _P], C.c_int),
    "b2k_gemm_noalloc_status": ([_I32], C.c_int),
    "b2k_gemm_set_chunk_split": ([C.c_int], C.c_int),
    "b2k_gemm_plan": ([_I32, _P, _P, _I64, _I64, _I64, _I64, _I64, _I32, C.POINTER(GemmPlan)], C.c_int),
    "b2k_row_softmax_f32_host": ([_P, _P, _P, _I64, _I64, _I64, _I64, _P], C.c_int),
    "b2k_pointwise_f32_host": ([_P, C.POINTER(PwProgram), C.POINTER(_P), _P, _I64, _P], C.c_int),
    "b2k_gemm_tf32x3_host": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _P, _I32, _P], C.c_int),
    "b2k_attention_tf32x3_host": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _I32, _P], C.c_int),
    "b2k_timing_enable": ([_P, C.c_int], C.c_int),
    "b2k_timing_select": ([_P, C.c_uint32], C.c_int),
    "b2k_set_pdl": ([C.c_int], C.c_int),
    "b2k_timing_read": ([_P, C.c_int, C.POINTER(C.c_double), C.POINTER(_I64)], C.c_int),
    "b2k_timing_reset": ([_P], C.c_int),
    "b2k_kernel_launches": ([C.c_void_p, C.POINTER(_I64)], C.c_int),
    "b2k_selftest_wait_timeout": ([C.c_void_p, _I64, C.c_void_p], C.c_int),
    "b2k_launch": ([C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p), C.c_int32, C.c_void_p], C.c_int),
    "b2k_mgpu_partition": ([_I64, _I32, _I32, _I64, C.POINTER(_I64), C.POINTER(_I64)], C.c_int),
    "b2k_mgpu_unique_id": ([_P], C.c_int),
    "b2k_mgpu_init": ([_P, _I32, _I32, _P, _I64, C.POINTER(_P)], C.c_int),
    "b2k_mgpu_destroy": ([_P], C.c_int),
    "b2k_mgpu_sync": ([_P, _P, _I64], C.c_int),
    "b2k_mgpu_gemm_tf32x3": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _P, _I32, _I32, _P], C.c_int),
    "b2k_mgpu_row_softmax_f32": ([_P, _P, _P, _I64, _I64, _I32, _P], C.c_int),
    "b2k_mgpu_pointwise_f32": ([_P, C.POINTER(PwProgram), C.POINTER(_P), _P, _I64, _I64, _I32, _P], C.c_int),
    "b2k_mgpu_attention_tf32x3": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _I32, _P], C.c_int),
}

PHASES = {"split": 0, "mma": 1, "pointwise": 2, "softmax": 3, "attention": 4, "rows": 5, "flash": 6}

_lock = threading.Lock()
_lib: C.CDLL | None = None


def library() -> C.CDLL:
    """Load ``libb200k.so`` once; raise if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIBRARY_PATH.exists():
                raise ImportError(f"{LIBRARY_PATH} is missing: build it with __graft_entry__.build() "
                                  "(the backend has no CPU fallback)")
            lib = C.CDLL(str(LIBRARY_PATH))
            for name, (argtypes, restype) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes, fn.restype = argtypes, restype
            _lib = lib
        return _lib


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def gemm_plan(sms: int, m: int, n: int, k: int, *, a: int = 256, b: int = 256, lda: int | None = None,
              ldb: int | None = None, b_layout: int = B_KN) -> dict:
    """The kernel path b2k_gemm_tf32x3 takes for these operands on a GPU of
    `sms` SMs (b2k_gemm_plan): host arithmetic, no GPU; `a` and `b` are
    addresses read only for their alignment."""
    lda = (m if b_layout & A_KM else k) if lda is None else lda
    ldb = (k if b_layout & B_NK else n) if ldb is None else ldb
    out = GemmPlan()
    status = library().b2k_gemm_plan(sms, a or None, b or None, m, n, k, lda, ldb, b_layout, C.byref(out))
    if status != B2K_OK:
        raise B2KError(status, "arguments b2k_gemm_tf32x3 refuses", "b2k_gemm_plan")
    return {"split_mode": out.split_mode, "tile_width": out.tile_width, "chunk_split": bool(out.chunk_split),
            "chunks": out.chunks}


def make_program(n_inputs: int, insns: list[tuple], result: int, broadcast=(), offsets=()) -> PwProgram:
    """Build a :class:`PwProgram`; ``insns`` are ``(opname, a, b, c, imm)`` tuples;
    ``offsets[r]`` shifts input stream r's window (element i reads i + offset)."""
    if n_inputs > PW_MAX_INPUTS or len(insns) > PW_MAX_INSNS:
        raise ValueError("pointwise program exceeds the kernel's register budget")
    prog = PwProgram()
    prog.n_inputs, prog.n_insns, prog.result = n_inputs, len(insns), result
    for i in range(PW_MAX_INPUTS):
        prog.broadcast[i] = 1 if i in tuple(broadcast) else 0
        prog.offset[i] = int(offsets[i]) if i < len(offsets) else 0
    for i, (op, a, b, c, imm) in enumerate(insns):
        prog.insns[i] = PwInsn(OPCODES[op] if isinstance(op, str) else int(op), a, b, c, float(imm))
    return prog


class BoundCall:
    """One library call with its arguments converted to C types once.

    Calling it re-issues the same call -- the same kernels on the same
    buffers, every step doing the full work -- without converting Python
    arguments again, which is most of the host cost of a short call made
    from Python.  Raises :class:`B2KError` on a failed status, like the
    methods of :class:`Context`.
    """

    def __init__(self, ctx: "Context", name: str, args: tuple, keep: tuple = ()):
        fn = getattr(ctx.lib, name)
        converted = [a if isinstance(a, (C._SimpleCData, C._Pointer, C.Array)) or type(a).__name__ == "CArgObject"
                     else t(a) for t, a in zip(fn.argtypes, args)]
        self._fn, self._args, self._keep = fn, tuple(converted), keep
        self._ctx, self._name = ctx, name

    def __call__(self) -> None:
        status = self._fn(*self._args)
        if status != B2K_OK:
            self._ctx.check(status, self._name)

    def with_stream(self, stream: int) -> "BoundCall":
        """The same call on another stream (every entry point takes its stream
        as the last argument), e.g. a stream being captured into a CUDA graph."""
        other = BoundCall.__new__(BoundCall)
        other._fn, other._ctx, other._name, other._keep = self._fn, self._ctx, self._name, (self._keep, self)
        other._args = self._args[:-1] + (_P(stream),)
        return other


class Context:
    """One ``b2k_ctx`` on one CUDA device (not thread-safe, like the C object)."""

    def __init__(self, device: int = 0):
        self.lib = library()
        handle = _P()
        status = self.lib.b2k_init(device, C.byref(handle))
        if status != B2K_OK:
            raise B2KError(status, "context creation failed (no sm_100 device?)", "b2k_init")
        self.handle, self.device = handle, device

    def close(self) -> None:
        if self.handle:
            self.lib.b2k_destroy(self.handle)
            self.handle = None

    def __enter__(self) -> "Context":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def check(self, status: int, call: str) -> None:
        if status != B2K_OK:
            reason = self.lib.b2k_last_error(self.handle) or b""
            raise B2KError(status, reason.decode(errors="replace"), call)

    @property
    def sm_count(self) -> int:
        return self.lib.b2k_sm_count(self.handle)

    # --- kernels (pointers are plain integers: device addresses) ----------
    def pointwise(self, program: PwProgram, inputs: list[int], out: int, n: int, stream: int = 0) -> None:
        arr = (_P * max(1, len(inputs)))(*inputs)
        self.check(self.lib.b2k_pointwise_f32(self.handle, C.byref(program), arr, out, n, stream),
                   "b2k_pointwise_f32")

    def row_softmax(self, x: int, y: int, rows: int, cols: int, ld_x: int | None = None,
                    ld_y: int | None = None, stream: int = 0) -> None:
        self.check(self.lib.b2k_row_softmax_f32(self.handle, x, y, rows, cols, ld_x or cols, ld_y or cols, stream),
                   "b2k_row_softmax_f32")

    def row_op(self, op: int, x: int, y: int, rows: int, cols: int, *, ld_x: int | None = None,
               ld_y: int | None = None, sum_div: float = 1.0, sum_div_ptr: int = 0, ms_div: float = 1.0,
               ms_div_ptr: int = 0, eps: float = 0.0, eps_ptr: int = 0, w: int = 0, stream: int = 0) -> None:
        params = RowParams(op, sum_div, sum_div_ptr or None, ms_div, ms_div_ptr or None, eps, eps_ptr or None,
                           w or None)
        self.check(self.lib.b2k_row_op_f32(self.handle, C.byref(params), x, y, rows, cols, ld_x or cols,
                                           ld_y or cols, stream), "b2k_row_op_f32")

    def axis_reduce(self, op: int, x: int, y: int, batch: int, s: int, cols: int, *, div: float = 1.0,
                    div_ptr: int = 0, stream: int = 0) -> None:
        """y[b][j] = fold over i < s of x[b][i][j] (ROW_SUM / ROW_MAX / ROW_MIN / ROW_PROD)."""
        self.check(self.lib.b2k_axis_reduce_f32(self.handle, op, x, y, batch, s, cols, div, div_ptr or None, stream),
                   "b2k_axis_reduce_f32")

    def selective_exp(self, x: int, y: int, n: int, stream: int = 0) -> None:
        self.check(self.lib.b2k_selective_exp_f32(self.handle, x, y, n, stream), "b2k_selective_exp_f32")

    def _gemm_args(self, a, b, c, m, n, k, b_layout=B_KN, lda=None, ldb=None, ldc=None, bias=0, relu=False,
                   stream=0) -> tuple:
        lda = (m if b_layout & A_KM else k) if lda is None else lda
        ldb = (k if b_layout & B_NK else n) if ldb is None else ldb
        ldc = n if ldc is None else ldc
        return (self.handle, a, b, c, m, n, k, lda, ldb, ldc, b_layout, bias or None, int(relu), stream)

    def gemm(self, a: int, b: int, c: int, m: int, n: int, k: int, *, b_layout: int = B_KN,
             lda: int | None = None, ldb: int | None = None, ldc: int | None = None,
             bias: int = 0, relu: bool = False, stream: int = 0) -> None:
        self.check(self.lib.b2k_gemm_tf32x3(*self._gemm_args(a, b, c, m, n, k, b_layout, lda, ldb, ldc, bias, relu,
                                                             stream)), "b2k_gemm_tf32x3")

    def gemm_scaled(self, a: int, b: int, c: int, m: int, n: int, k: int, *, div_ptr: int = 0,
                    div_value: float = 1.0, b_layout: int = B_KN, lda: int | None = None, ldb: int | None = None,
                    ldc: int | None = None, bias: int = 0, relu: bool = False, stream: int = 0) -> None:
        """C = relu?((A B) / div + bias), div = *div_ptr (device) or div_value."""
        args = self._gemm_args(a, b, c, m, n, k, b_layout, lda, ldb, ldc, bias, relu, stream)
        self.check(self.lib.b2k_gemm_tf32x3_scaled(*args[:-1], div_ptr or None, div_value, args[-1]),
                   "b2k_gemm_tf32x3_scaled")

    def gemm_batched(self, a: int, b: int, c: int, batch: int, m: int, n: int, k: int, *, b_layout: int = B_KN,
                     bias: int = 0, relu: bool = False, stream: int = 0) -> None:
        """C[i] = relu?(A[i] B[i] + bias) over contiguous [batch][rows][cols] operands."""
        ldb = n if b_layout == B_KN else k
        self.check(self.lib.b2k_gemm_tf32x3_batched(self.handle, a, b, c, batch, m, n, k, k, ldb, n, m * k, n * k,
                                                    m * n, b_layout, bias or None, int(relu), stream),
                   "b2k_gemm_tf32x3_batched")

    def gemm_call(self, a: int, b: int, c: int, m: int, n: int, k: int, **kw) -> "BoundCall":
        """:meth:`gemm` with its arguments converted once (see :class:`BoundCall`)."""
        return BoundCall(self, "b2k_gemm_tf32x3", self._gemm_args(a, b, c, m, n, k, **kw))

    def _attention_args(self, q, k, v, o, bh, s_q, s_kv, d, dv, scale=None, scale_ptr=0, k_layout=K_SD,
                        stream=0) -> tuple:
        div = float(d) ** 0.5 if scale is None else float(scale)
        return (self.handle, q, k, v, o, bh, s_q, s_kv, d, dv, div, scale_ptr or None, k_layout, stream)

    def attention(self, q: int, k: int, v: int, o: int, bh: int, s_q: int, s_kv: int, d: int, dv: int, *,
                  scale: float | None = None, scale_ptr: int = 0, k_layout: int = K_SD, stream: int = 0) -> None:
        """O = softmax(Q K^T / scale) V per head; scale defaults to sqrt(d)."""
        self.check(self.lib.b2k_attention_tf32x3(*self._attention_args(q, k, v, o, bh, s_q, s_kv, d, dv, scale,
                                                                       scale_ptr, k_layout, stream)),
                   "b2k_attention_tf32x3")

    def attention_call(self, q: int, k: int, v: int, o: int, bh: int, s_q: int, s_kv: int, d: int, dv: int,
                       **kw) -> "BoundCall":
        """:meth:`attention` with its arguments converted once."""
        return BoundCall(self, "b2k_attention_tf32x3", self._attention_args(q, k, v, o, bh, s_q, s_kv, d, dv, **kw))

    def row_softmax_call(self, x: int, y: int, rows: int, cols: int, ld_x: int | None = None,
                         ld_y: int | None = None, stream: int = 0) -> "BoundCall":
        """:meth:`row_softmax` with its arguments converted once."""
        return BoundCall(self, "b2k_row_softmax_f32", (self.handle, x, y, rows, cols, ld_x or cols, ld_y or cols,
                                                        stream))

    def pointwise_call(self, program: PwProgram, inputs: list[int], out: int, n: int,
                       stream: int = 0) -> "BoundCall":
        """:meth:`pointwise` with its arguments converted once."""
        arr = (_P * max(1, len(inputs)))(*inputs)
        return BoundCall(self, "b2k_pointwise_f32", (self.handle, C.byref(program), arr, out, n, stream),
                         keep=(program, arr))

    # --- pipelined host-array calls: the same operations on HOST pointers, with
    # the copies in, the kernels and the copies out overlapped slab by slab.
    def row_softmax_host(self, x: int, y: int, rows: int, cols: int, ld_x: int | None = None,
                         ld_y: int | None = None, stream: int = 0) -> None:
        self.check(self.lib.b2k_row_softmax_f32_host(self.handle, x, y, rows, cols, ld_x or cols, ld_y or cols,
                                                     stream), "b2k_row_softmax_f32_host")

    def pointwise_host(self, program: PwProgram, inputs: list[int], out: int, n: int, stream: int = 0) -> None:
        arr = (_P * max(1, len(inputs)))(*inputs)
        self.check(self.lib.b2k_pointwise_f32_host(self.handle, C.byref(program), arr, out, n, stream),
                   "b2k_pointwise_f32_host")

    def gemm_host(self, a: int, b: int, c: int, m: int, n: int, k: int, *, b_layout: int = B_KN,
                  lda: int | None = None, ldb: int | None = None, ldc: int | None = None,
                  bias: int = 0, relu: bool = False, stream: int = 0) -> None:
        self.check(self.lib.b2k_gemm_tf32x3_host(*self._gemm_args(a, b, c, m, n, k, b_layout, lda, ldb, ldc, bias,
                                                                  relu, stream)), "b2k_gemm_tf32x3_host")

    def attention_host(self, q: int, k: int, v: int, o: int, bh: int, s_q: int, s_kv: int, d: int, dv: int, *,
                       scale: float | None = None, k_layout: int = K_SD, stream: int = 0) -> None:
        div = float(d) ** 0.5 if scale is None else float(scale)
        self.check(self.lib.b2k_attention_tf32x3_host(self.handle, q, k, v, o, bh, s_q, s_kv, d, dv, div, k_layout,
                                                      stream), "b2k_attention_tf32x3_host")

    def timing(self, on: bool, phases: list[str] | None = None) -> None:
        """Enable per-phase event timing, for `phases` only when given."""
        mask = 0xFFFFFFFF if phases is None else sum(1 << PHASES[p] for p in phases)
        self.check(self.lib.b2k_timing_select(self.handle, mask), "b2k_timing_select")
        self.check(self.lib.b2k_timing_enable(self.handle, int(on)), "b2k_timing_enable")

    def timing_read(self, phase: str) -> tuple[float, int]:
        """(total milliseconds, launches) recorded for one phase since the last reset."""
        ms, count = C.c_double(), _I64()
        self.check(self.lib.b2k_timing_read(self.handle, PHASES[phase], C.byref(ms), C.byref(count)),
                   "b2k_timing_read")
        return ms.value, count.value

    def timing_reset(self) -> None:
        self.check(self.lib.b2k_timing_reset(self.handle), "b2k_timing_reset")

    def set_gemm_variant(self, variant: int) -> None:
        self.check(self.lib.b2k_gemm_set_variant(variant), "b2k_gemm_set_variant")

    def launch(self, desc: KernelDesc, arg_values: list, stream: int = 0) -> None:
        """b2k_launch with the positional arguments in arg_order: ints are device
        addresses, floats are f32 scalars (each passed as a pointer to its value,
        the cuLaunchKernel params convention)."""
        slots = [C.c_uint64(v) if isinstance(v, int) else C.c_float(v) for v in arg_values]
        params = (C.c_void_p * max(1, len(slots)))(*[C.cast(C.pointer(x), C.c_void_p) for x in slots])
        self.check(self.lib.b2k_launch(self.handle, C.byref(desc), params, len(slots), stream), "b2k_launch")

    def kernel_launches(self) -> int:
        """Kernels this context has enqueued since it was created."""
        count = _I64()
        self.check(self.lib.b2k_kernel_launches(self.handle, C.byref(count)), "b2k_kernel_launches")
        return int(count.value)

    def set_gemm_chunk_split(self, mode: int) -> None:
        """0 = never split the pre-pass GEMM over K chunks, 1 (default) = where
        estimated faster, 2 = wherever it applies (same bits in every mode)."""
        self.check(self.lib.b2k_gemm_set_chunk_split(int(mode)), "b2k_gemm_set_chunk_split")

    def set_gemm_fused_split(self, mode: int) -> None:
        """0 = pre-pass split of A and B; 3 = A split in-kernel into TMEM (direct);
        2 = B split in-kernel into TMEM, C^T = B^T A^T (transposed); 1 (default)
        = whichever of the three the estimate says is fastest."""
        self.check(self.lib.b2k_gemm_set_fused_split(int(mode)), "b2k_gemm_set_fused_split")

    def set_pdl(self, on: bool) -> None:
        """Programmatic dependent launch between a call's kernels (process-wide, default on)."""
        self.check(self.lib.b2k_set_pdl(int(bool(on))), "b2k_set_pdl")

    def sync(self, stream: int = 0) -> None:
        self.check(self.lib.b2k_stream_sync(self.handle, stream), "b2k_stream_sync")

    # --- memory helpers (used by callers without PyTorch) -------------------
    def malloc(self, nbytes: int) -> int:
        ptr = _P()
        self.check(self.lib.b2k_malloc(self.handle, C.byref(ptr), nbytes), "b2k_malloc")
        return ptr.value or 0

    def host_alloc(self, nbytes: int) -> int:
        ptr = _P()
        self.check(self.lib.b2k_host_alloc(self.handle, C.byref(ptr), nbytes), "b2k_host_alloc")
        return ptr.value or 0

    def host_free(self, ptr: int) -> None:
        self.check(self.lib.b2k_host_free(self.handle, ptr), "b2k_host_free")

    def free(self, ptr: int) -> None:
        self.check(self.lib.b2k_free(self.handle, ptr), "b2k_free")

    def htod(self, dst: int, src: int, nbytes: int, stream: int = 0) -> None:
        self.check(self.lib.b2k_memcpy_htod(self.handle, dst, src, nbytes, stream), "b2k_memcpy_htod")

    def dtoh(self, dst: int, src: int, nbytes: int, stream: int = 0) -> None:
        self.check(self.lib.b2k_memcpy_dtoh(self.handle, dst, src, nbytes, stream), "b2k_memcpy_dtoh")

    def memset(self, dst: int, value: int, nbytes: int, stream: int = 0) -> None:
        self.check(self.lib.b2k_memset(self.handle, dst, value, nbytes, stream), "b2k_memset")


# --- multi-GPU (b2k_mgpu_*) ---------------------------------------------------
def mgpu_partition(units: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """(start, count) of ``rank``'s shard, computed by the library
    (``b2k_mgpu_partition``; host arithmetic, no device needed)."""
    start, count = _I64(), _I64()
    status = library().b2k_mgpu_partition(units, world, rank, align, C.byref(start), C.byref(count))
    if status != B2K_OK:
        raise B2KError(status, "bad partition request", "b2k_mgpu_partition")
    return start.value, count.value


def mgpu_unique_id() -> bytes:
    """The communicator's rendezvous token (made on one rank, given to all)."""
    buf = C.create_string_buffer(MGPU_ID_BYTES)
    status = library().b2k_mgpu_unique_id(buf)
    if status != B2K_OK:
        raise B2KError(status, "NCCL unavailable or failed to make an id", "b2k_mgpu_unique_id")
    return buf.raw


class MultiGpu:
    """One rank of a ``b2k_mgpu`` communicator, bound to a :class:`Context`.

    Every method takes this rank's shard of the inputs (device addresses) and
    leaves the whole output on every rank; see include/b200k.h."""

    def __init__(self, ctx: Context, world: int, rank: int, uid: bytes, timeout_ms: int = 60000):
        if len(uid) != MGPU_ID_BYTES:
            raise ValueError("the unique id is 128 bytes")
        self.ctx, self.world, self.rank = ctx, world, rank
        self._uid = C.create_string_buffer(uid, MGPU_ID_BYTES)
        handle = _P()
        ctx.check(ctx.lib.b2k_mgpu_init(ctx.handle, world, rank, self._uid, timeout_ms, C.byref(handle)),
                  "b2k_mgpu_init")
        self.handle = handle

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.ctx.lib.b2k_mgpu_destroy(self.handle)
            self.handle = None

    def __enter__(self) -> "MultiGpu":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def _call(self, name: str, *args) -> None:
        self.ctx.check(getattr(self.ctx.lib, name)(self.handle, *args), name)

    def sync(self, stream: int = 0, timeout_ms: int = 60000) -> None:
        self._call("b2k_mgpu_sync", stream, timeout_ms)

    def gemm(self, a_rows: int, b: int, c: int, m: int, n: int, k: int, *, align: int = 1, b_layout: int = B_KN,
             bias: int = 0, relu: bool = False, panels: int = 1, stream: int = 0) -> None:
        self._call("b2k_mgpu_gemm_tf32x3", a_rows, b or None, c, m, n, k, align, b_layout, bias or None, int(relu),
                   panels, stream)

    def row_softmax(self, x_rows: int, y: int, rows: int, cols: int, *, pieces: int = 1, stream: int = 0) -> None:
        self._call("b2k_mgpu_row_softmax_f32", x_rows or None, y, rows, cols, pieces, stream)

    def pointwise(self, program: PwProgram, inputs: list[int], out: int, n: int, *, align: int = 1,
                  pieces: int = 1, stream: int = 0) -> None:
        ptrs = (_P * max(1, len(inputs)))(*inputs)
        self._call("b2k_mgpu_pointwise_f32", C.byref(program), ptrs, out, n, align, pieces, stream)

    def attention(self, q: int, k: int, v: int, o: int, bh: int, s_q: int, s_kv: int, d: int, dv: int, *,
                  scale_div: float | None = None, pieces: int = 1, stream: int = 0) -> None:
        scale = float(d) ** 0.5 if scale_div is None else float(scale_div)
        self._call("b2k_mgpu_attention_tf32x3", q or None, k or None, v or None, o, bh, s_q, s_kv, d, dv, scale,
                   pieces, stream)
