"""
NVFP4 linear layers on B200 (sm_100a) -- drop-in for the ``fp4_gemm`` module
of VincentKaufmann/fp4-gemm-blackwell (fp4_gemm.py in that project).

Same public names, argument meaning, return values and errors:

    fp4_matmul(A, B, C=None, alpha=1.0, beta=0.0)  D = alpha*q(A) @ q(B)^T + beta*C
    fp4_linear(x, weight, bias=None)              F.linear with FP4 operands
    FP4WeightCache(weight, bias=None)             quantize once, .forward(x, sync=True)
    fp4_quantize(weight, bias=None)               -> FP4WeightCache
    fp4_cached_matmul(A, cache), fp4_cached_linear(x, cache)
    sync(), prealloc(max_M, max_N, max_K), cleanup(), SF_VEC_SIZE

The work runs in ``libfp4gemm.so`` (beside this file, loaded through ctypes with
tensors passed by pointer, as the reference does at fp4_gemm.py:26-27): a
vectorised BF16->NVFP4 quantizer and a tcgen05 block-scaled GEMM.  Results
equal the reference's: the reference zero-pads M, N, K to multiples of 128 and
slices the output afterwards; here the kernels read the unpadded tensors
(zeros outside, same quantized bytes) and write only the valid [M, N] block,
so the pad and unpad copies disappear.  The bias is added inside the GEMM
epilogue with the reference's rounding order (BF16 product, then a BF16 add).
Work is issued on PyTorch's current CUDA stream; ``sync=True`` and
``fp4_matmul`` synchronise the device exactly where the reference does.

There is no fallback: importing this module fails if the library is missing.
"""

import ctypes
import math
import os

import torch

_lib_path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libfp4gemm.so")
if not os.path.exists(_lib_path):
    raise ImportError(
        f"{_lib_path} is missing; build it with `python {os.path.join(os.path.dirname(_lib_path), 'build.py')}`")
_lib = ctypes.CDLL(_lib_path)

_vp, _i, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def _bind(name, restype, argtypes):
    fn = getattr(_lib, name)
    fn.restype = restype
    fn.argtypes = argtypes
    return fn


# Reference ABI (fp4_gemm.py:30-84 of the reference binds the same signatures).
_bind("fp4_gemm_sf_vec_size", _i, [])
_bind("fp4_gemm_init", _i, [_i, _i, _i])
_bind("fp4_gemm_run", _i, [_vp, _vp, _vp, _vp, _i, _i, _i, _f, _f])
_bind("fp4_gemm_cleanup", None, [])
_bind("fp4_gemm_prealloc", _i, [_i, _i, _i])
_bind("fp4_gemm_sync", None, [])
_bind("fp4_quantize_weights", _vp, [_vp, _i, _i])
_bind("fp4_weight_cache_free", None, [_vp])
_bind("fp4_weight_cache_N", _i, [_vp])
_bind("fp4_weight_cache_K", _i, [_vp])
_bind("fp4_weight_cache_fp4_ptr", _vp, [_vp])
_bind("fp4_weight_cache_sf_ptr", _vp, [_vp])
_bind("fp4_gemm_run_cached", _i, [_vp, _vp, _vp, _vp, _i, _f, _f])
# Additive ABI.
_bind("fp4b_version", _i, [])
_bind("fp4b_gemm_tile_width", _i, [_i, _i, _i, _i])
_bind("fp4b_selftest_bounded_wait", _i, [_i, _vp])
_bind("fp4b_last_error", ctypes.c_char_p, [])
_bind("fp4b_device_error", _i, [_i])
_bind("fp4b_quantize", _i, [_vp, _i, _i, _i, _vp, _vp, _i, _i, _vp])
_bind("fp4b_gemm_prequant", _i, [_vp, _vp, _i, _i, _vp, _vp, _i, _i, _i, _vp, _i, _vp, _i, _vp, _f, _f, _vp])
_bind("fp4b_run_cached_ex", _i, [_vp, _i, _i, _i, _vp, _i, _vp, _i, _vp, _i, _vp, _f, _f, _vp])
_bind("fp4b_run_ex", _i, [_vp, _i, _i, _i, _vp, _i, _i, _vp, _i, _vp, _i, _vp, _f, _f, _vp])
_bind("fp4b_quantize_weights_ex", _vp, [_vp, _i, _i, _i, _vp, _i])
_bind("fp4b_weight_cache_slice", _vp, [_vp, _i, _i])
_bind("fp4b_weight_cache_set_alpha", _i, [_vp, _f])
_bind("fp4b_weight_cache_alpha", _f, [_vp])
_bind("fp4b_weight_cache_export", _i, [_vp, _vp, _vp, _vp])
_bind("fp4b_weight_cache_import", _vp, [_vp, _vp, _i, _i, _vp])
_bind("fp4b_run_cached_peers", _i, [_vp, _i, _i, _i, _vp, _i, _vp, _i, ctypes.POINTER(_vp), _i, _vp, _vp])
_bind("fp4b_ipc_get_handle", _i, [_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_long)])
_bind("fp4b_ipc_open_handle", _vp, [ctypes.c_char_p, ctypes.c_long])
_bind("fp4b_ipc_close", _i, [_vp, ctypes.c_long])
_bind("fp4b_mma_rate", _i, [_i, _i, _i, _i, _i, ctypes.POINTER(_i), _vp])
_bind("fp4b_peer_barrier", _i, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_i), _i, _i, ctypes.c_ulonglong, _vp])
_bind("fp4b_copy2d", _i, [_vp, ctypes.c_long, _vp, ctypes.c_long, ctypes.c_long, ctypes.c_long, _vp])

# Query scale factor vector size
SF_VEC_SIZE = _lib.fp4_gemm_sf_vec_size()


_SIDE_STREAMS = {}  # device -> (host-to-device, device-to-host) copy streams for forward_host


def _chunk_schedule(m: int, chunk_rows: int) -> list:
    """Row counts of forward_host's chunks.  Equal chunks of chunk_rows: on B200
    with PCIe Gen5 a tail of halving chunks (512, 256, 128, ...) measured slower
    than equal 512-row chunks, whose copies already hide the per-chunk GEMMs."""
    return [min(chunk_rows, m - r) for r in range(0, m, chunk_rows)]


# Largest UE4M3 block scale the quantizer produces (the clamp of fp4_gemm_lib.cu:128-164).
_UE4M3_MAX = 480.0


def global_weight_scale(amax: float) -> float:
    """Power of two s for two-level NVFP4 weights: quantizing weight * s puts the
    largest block scale (|w|max * s / 6) at or just below the UE4M3 maximum 480,
    so that the block scales of small-magnitude weights use UE4M3's normal range
    (rounded) instead of its subnormals (truncated).  A power of two keeps
    weight * s exact in BF16 and 1 / s exact in the GEMM's alpha.  1 for a zero
    or non-finite |w|max."""
    if not (amax > 0.0) or amax != amax or amax == float("inf"):
        return 1.0
    return 2.0 ** math.floor(math.log2(6.0 * _UE4M3_MAX / amax))


def _pad_to_multiple(x: int, m: int) -> int:
    """Smallest multiple of m that is >= x (the reference pads M, N, K to 128)."""
    return -(-x // m) * m


def _stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _last_error() -> str:
    msg = _lib.fp4b_last_error()
    return msg.decode() if msg else ""


def _rows_view(t: torch.Tensor):
    """(tensor, row stride) with unit column stride; copies only if needed."""
    if t.dim() == 2 and t.stride(1) == 1 and t.stride(0) >= t.shape[1]:
        return t, t.stride(0)
    t = t.contiguous()
    return t, t.shape[1]


def fp4_matmul(
    A: torch.Tensor,
    B: torch.Tensor,
    C: torch.Tensor = None,
    alpha: float = 1.0,
    beta: float = 0.0,
) -> torch.Tensor:
    """
    Dynamic NVFP4 product: both operands are quantized on every call.

    D = alpha * q(A) @ q(B)^T + beta * C, where q() is the NVFP4 quantizer
    (E2M1 values, one UE4M3 scale per 16 elements along K) and the product is
    accumulated in fp32 by the tcgen05 tensor cores and rounded to BF16.

    A is [M, K] or a batch [b, M, K] of activations, B is [N, K] (a weight in
    F.linear layout), C an optional [M, N] term scaled by beta; all BF16 CUDA
    tensors (other float types are cast to BF16 first).  The result is a BF16
    [M, N] tensor, or [b, M, N] for a batched A.

    M, N and K need not be multiples of 128: the quantized operands equal the
    reference's zero-padded ones, without the padding copies.  The device is
    synchronised before returning, as the reference's fp4_gemm_run does.
    """
    batched = A.dim() == 3
    if batched:
        batch_size = A.shape[0]
        A = A.reshape(-1, A.shape[-1])

    assert A.dim() == 2, f"A must be 2D [M, K] or 3D [batch, M, K], got shape {A.shape}"
    assert B.dim() == 2, f"B must be 2D [N, K], got shape {B.shape}"
    assert A.shape[1] == B.shape[1], f"K mismatch: A has K={A.shape[1]}, B has K={B.shape[1]}"
    assert A.is_cuda and B.is_cuda, "Both tensors must be on CUDA"

    M_orig, K_orig = A.shape
    N_orig = B.shape[0]

    if A.dtype != torch.bfloat16:
        A = A.to(torch.bfloat16)
    if B.dtype != torch.bfloat16:
        B = B.to(torch.bfloat16)

    D = torch.empty(M_orig, N_orig, dtype=torch.bfloat16, device=A.device)
    if M_orig > 0 and N_orig > 0:
        if K_orig == 0:
            D.zero_()
            if C is not None and beta != 0.0:
                D = (beta * C.to(torch.bfloat16).float()).to(torch.bfloat16).reshape(M_orig, N_orig)
        else:
            A, lda = _rows_view(A)
            B, ldb = _rows_view(B)
            c_ptr, ldc = None, 0
            if C is not None:
                if C.dtype != torch.bfloat16:
                    C = C.to(torch.bfloat16)
                C = C.expand(M_orig, N_orig) if C.shape != (M_orig, N_orig) else C
                C = C.contiguous()
                c_ptr, ldc = C.data_ptr(), N_orig
            with torch.cuda.device(A.device):
                rc = _lib.fp4b_run_ex(A.data_ptr(), M_orig, K_orig, lda, B.data_ptr(), N_orig, ldb, c_ptr, ldc,
                                      D.data_ptr(), N_orig, None, float(alpha), float(beta), _stream_ptr(A.device))
                if rc != 0:
                    raise RuntimeError(f"fp4_gemm_run failed with error code {rc} ({_last_error()})")
                _lib.fp4_gemm_sync()

    if batched:
        D = D.reshape(batch_size, -1, N_orig)

    return D


def fp4_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor = None) -> torch.Tensor:
    """
    F.linear(x, weight, bias) computed as a dynamic NVFP4 product.

    x is [..., K]; weight is [N, K]; bias, when given, is [N] and is added to
    the BF16 product afterwards (a second BF16 rounding, as in the reference).
    Returns [..., N].
    """
    orig_shape = x.shape
    x_2d = x.reshape(-1, x.shape[-1])

    out = fp4_matmul(x_2d, weight)

    if bias is not None:
        out = out + bias.unsqueeze(0)

    out = out.reshape(*orig_shape[:-1], weight.shape[0])
    return out


def sync():
    """Wait for all queued work on the current device (cudaDeviceSynchronize);
    use it after a run of forward(..., sync=False) calls."""
    _lib.fp4_gemm_sync()


def prealloc(max_M: int, max_N: int, max_K: int):
    """
    Size the library's per-device scratch for the largest problem to come
    (rows of activations, output features, input features; each rounded up to
    128 here), so that later calls do not grow it while a model is running.
    """
    rc = _lib.fp4_gemm_prealloc(*(_pad_to_multiple(v, 128) for v in (max_M, max_N, max_K)))
    if rc != 0:
        raise RuntimeError(f"fp4_gemm_prealloc failed with code {rc}")


def cleanup():
    """Free the scratch buffers the library holds on the current device."""
    _lib.fp4_gemm_cleanup()


class FP4WeightCache:
    """
    A weight quantized to NVFP4 once and kept on the GPU.

    Each ``forward(x)`` quantizes only the activations and multiplies them
    with the stored weight (plus the bias, when one was given).  Free the
    device memory with ``free()``, or use the object in a ``with`` block.

    The stored bytes (``fp4_bytes`` of packed E2M1 for the weight padded to
    multiples of 128 in both dimensions, then ``sf_bytes`` of scales) are the
    ones the reference's cache holds for the same weight.
    """

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor = None, global_scale: bool = False):
        """
        weight: the [N, K] CUDA weight (F.linear layout; cast to BF16).
        bias: optional [N] tensor added to every output row.
        global_scale: two-level NVFP4, not in the reference and off by default
            (off keeps the reference's bytes).  The cache then holds
            weight * s, s the power of two ``global_weight_scale(|weight|max)``,
            and every GEMM with it is multiplied by 1 / s.  This helps weights
            of small magnitude (e.g. N(0, 0.02)), whose block scales would
            otherwise fall among UE4M3's truncated subnormals.
        """
        self._handle = None
        assert weight.dim() == 2, f"Weight must be 2D [N, K], got {weight.shape}"
        assert weight.is_cuda, "Weight must be on CUDA"

        self.N_orig = weight.shape[0]
        self.K_orig = weight.shape[1]
        self.bias = bias

        # Padded (cached) shape, multiples of 128
        self.N = _pad_to_multiple(self.N_orig, 128)
        self.K = _pad_to_multiple(self.K_orig, 128)
        self.padded = (self.N != self.N_orig or self.K != self.K_orig)

        if weight.dtype != torch.bfloat16:
            weight = weight.to(torch.bfloat16)
        self.global_scale = 1.0
        if global_scale:
            self.global_scale = global_weight_scale(float(weight.abs().max().float()))
            if self.global_scale != 1.0:
                weight = (weight.float() * self.global_scale).to(torch.bfloat16)  # exact: a power of two
        weight, ldw = _rows_view(weight)
        self.device = weight.device

        with torch.cuda.device(weight.device):
            handle = _lib.fp4b_quantize_weights_ex(weight.data_ptr(), self.N_orig, self.K_orig, ldw,
                                                   _stream_ptr(weight.device), 1)
        if not handle:
            raise RuntimeError("fp4_quantize_weights failed")
        self._handle = handle
        if self.global_scale != 1.0 and _lib.fp4b_weight_cache_set_alpha(handle, 1.0 / self.global_scale) != 0:
            raise RuntimeError(f"fp4b_weight_cache_set_alpha failed ({_last_error()})")

        # Memory tracking
        self.fp4_bytes = self.N * self.K // 2
        # Scale factors: 1 byte per 16 elements
        self.sf_bytes = self.N * (self.K // 16)

    @classmethod
    def _from_handle(cls, handle: int, n_orig: int, k_orig: int, device, bias=None):
        obj = cls.__new__(cls)
        obj._handle = handle
        obj.N_orig, obj.K_orig, obj.bias = n_orig, k_orig, bias
        obj.N = _lib.fp4_weight_cache_N(handle)
        obj.K = _lib.fp4_weight_cache_K(handle)
        obj.padded = (obj.N != n_orig or obj.K != k_orig)
        obj.device = device
        w_alpha = _lib.fp4b_weight_cache_alpha(handle)
        obj.global_scale = 1.0 / w_alpha if w_alpha > 0 else 1.0
        obj.fp4_bytes = obj.N * obj.K // 2
        obj.sf_bytes = obj.N * (obj.K // 16)
        return obj

    def forward(self, x: torch.Tensor, sync: bool = True) -> torch.Tensor:
        """
        y = q(x) @ W^T (+ bias) for activations x [..., K] on the cache's
        device; returns [..., N].  The work is queued on the current stream;
        with sync=True (the reference's default) the device is synchronised
        before returning, so pass sync=False for back-to-back calls.
        """
        if self._handle is None:
            raise RuntimeError("FP4WeightCache has been freed")

        orig_shape = x.shape
        x_2d = x.reshape(-1, x.shape[-1])

        M_orig = x_2d.shape[0]
        K_in = x_2d.shape[1]

        if K_in != self.K_orig:
            raise ValueError(f"Input K={K_in} doesn't match weight K={self.K_orig}")

        if x_2d.dtype != torch.bfloat16:
            x_2d = x_2d.to(torch.bfloat16)

        bias = self.bias
        fuse_bias = bias is not None and bias.dtype == torch.bfloat16 and bias.is_cuda
        D = torch.empty(M_orig, self.N_orig, dtype=torch.bfloat16, device=x_2d.device)
        if M_orig > 0:
            x_2d, lda = _rows_view(x_2d)
            b_ptr = None
            if fuse_bias:
                bias = bias.reshape(-1).contiguous()
                b_ptr = bias.data_ptr()
            with torch.cuda.device(x_2d.device):
                rc = _lib.fp4b_run_cached_ex(x_2d.data_ptr(), M_orig, K_in, lda, self._handle, self.N_orig, None, 0,
                                             D.data_ptr(), self.N_orig, b_ptr, 1.0, 0.0, _stream_ptr(x_2d.device))
            if rc != 0:
                raise RuntimeError(f"fp4_gemm_run_cached failed with error code {rc} ({_last_error()})")

        # Sync if requested (skip for pipelined calls)
        if sync:
            _lib.fp4_gemm_sync()

        if self.bias is not None and not fuse_bias:
            D = D + self.bias.unsqueeze(0)

        D = D.reshape(*orig_shape[:-1], self.N_orig)
        return D

    def forward_host(self, x: torch.Tensor, out: torch.Tensor = None, chunk_rows: int = 512) -> torch.Tensor:
        """
        Cached linear on host buffers: output = x @ cached_weight.T + bias with
        x and the result in (pinned) CPU memory.

        Rows are processed in chunks of ``chunk_rows`` (a multiple of 128):
        the host-to-device copy of chunk c+1 runs on one side stream while
        chunk c is quantized and multiplied on the caller's current stream and
        chunk c-1 is copied back on another side stream, so the PCIe transfers
        in both directions overlap each other and the GPU work; only the last
        chunk's GEMM and copy back follow the last input copy.  The side streams
        start after the work already queued on the current stream, and the
        current stream waits for the last copy back, so the call is ordered
        like any other stream operation; pass ``out`` (pinned, [..., N] BF16)
        to reuse an output buffer, and synchronize before reading it.

        Args:
            x: Input activation [..., K] BF16 in CPU memory (pinned for overlap)
            out: Optional CPU output [..., N] BF16
            chunk_rows: rows per pipelined chunk

        Returns:
            CPU tensor [..., N] (``out`` when given)
        """
        if self._handle is None:
            raise RuntimeError("FP4WeightCache has been freed")
        if x.is_cuda:
            raise ValueError("forward_host takes a CPU tensor; use forward for CUDA tensors")
        if chunk_rows <= 0 or chunk_rows % 128:
            raise ValueError("chunk_rows must be a positive multiple of 128")
        orig_shape = x.shape
        x_2d = x.reshape(-1, x.shape[-1])
        if x_2d.shape[1] != self.K_orig:
            raise ValueError(f"Input K={x_2d.shape[1]} doesn't match weight K={self.K_orig}")
        if x_2d.dtype != torch.bfloat16:
            x_2d = x_2d.to(torch.bfloat16)
        x_2d = x_2d.contiguous()
        M = x_2d.shape[0]
        if out is None:
            out = torch.empty(*orig_shape[:-1], self.N_orig, dtype=torch.bfloat16,
                              pin_memory=torch.cuda.is_available())
        if out.is_cuda or out.dtype != torch.bfloat16 or out.numel() != M * self.N_orig or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous CPU BF16 tensor of {M * self.N_orig} elements")
        out_2d = out.view(M, self.N_orig)
        if M == 0:
            return out

        dev = self.device
        cur = torch.cuda.current_stream(dev)
        h2d, d2h = self._side_streams()
        xd, yd = self._host_staging(M)
        bias = self.bias
        fuse_bias = bias is not None and bias.dtype == torch.bfloat16 and bias.is_cuda
        b_ptr = None
        if fuse_bias:
            bias = bias.reshape(-1).contiguous()
            b_ptr = bias.data_ptr()
        h2d.wait_stream(cur)
        d2h.wait_stream(cur)
        sptr = cur.cuda_stream
        with torch.cuda.device(dev):
            r1 = 0
            for rows in _chunk_schedule(M, chunk_rows):
                r0, r1 = r1, r1 + rows
                with torch.cuda.stream(h2d):
                    xd[r0:r1].copy_(x_2d[r0:r1], non_blocking=True)
                cur.wait_stream(h2d)
                rc = _lib.fp4b_run_cached_ex(xd[r0:r1].data_ptr(), r1 - r0, self.K_orig, self.K_orig, self._handle,
                                             self.N_orig, None, 0, yd[r0:r1].data_ptr(), self.N_orig, b_ptr, 1.0,
                                             0.0, sptr)
                if rc != 0:
                    raise RuntimeError(f"fp4_gemm_run_cached failed with error code {rc} ({_last_error()})")
                if self.bias is not None and not fuse_bias:
                    yd[r0:r1] += self.bias.to(device=dev, dtype=torch.bfloat16).unsqueeze(0)
                d2h.wait_stream(cur)
                with torch.cuda.stream(d2h):
                    out_2d[r0:r1].copy_(yd[r0:r1], non_blocking=True)
        cur.wait_stream(d2h)
        return out

    def _side_streams(self):
        st = _SIDE_STREAMS.get(self.device)
        if st is None:
            st = (torch.cuda.Stream(self.device), torch.cuda.Stream(self.device))
            _SIDE_STREAMS[self.device] = st
        return st

    def _host_staging(self, m: int):
        """Device staging for forward_host: [m, K] input and [m, N] output, grow-only."""
        st = getattr(self, "_staging", None)
        if st is None or st[0].shape[0] < m:
            rows = _pad_to_multiple(max(m, 128), 128)
            st = (torch.empty(rows, self.K_orig, dtype=torch.bfloat16, device=self.device),
                  torch.empty(rows, self.N_orig, dtype=torch.bfloat16, device=self.device))
            self._staging = st
        return st

    def shard(self, row0: int, rows: int, bias=None) -> "FP4WeightCache":
        """A cache viewing rows [row0, row0+rows) of this one (multiples of 128), for N-sharding."""
        h = _lib.fp4b_weight_cache_slice(self._handle, row0, rows)
        if not h:
            raise RuntimeError(f"fp4b_weight_cache_slice failed ({_last_error()})")
        view = FP4WeightCache._from_handle(h, rows, self.K_orig, self.device, bias)
        view._parent = self  # keep the owner alive
        return view

    def state_dict(self) -> dict:
        """Serialisable payload: the cached bytes (device uint8 tensors) and shapes.

        ``FP4WeightCache.from_state_dict`` rebuilds the cache without
        re-quantizing (the reference re-quantizes at every model load)."""
        if self._handle is None:
            raise RuntimeError("FP4WeightCache has been freed")
        fp4 = torch.empty(self.N, self.K // 2, dtype=torch.uint8, device=self.device)
        sf = torch.empty(self.N * self.K // 16, dtype=torch.uint8, device=self.device)
        with torch.cuda.device(self.device):
            rc = _lib.fp4b_weight_cache_export(self._handle, fp4.data_ptr(), sf.data_ptr(), _stream_ptr(self.device))
        if rc != 0:
            raise RuntimeError(f"fp4b_weight_cache_export failed ({_last_error()})")
        return {"fp4": fp4, "sf": sf, "N_orig": self.N_orig, "K_orig": self.K_orig, "bias": self.bias,
                "global_scale": self.global_scale}

    @classmethod
    def from_state_dict(cls, sd: dict, device=None) -> "FP4WeightCache":
        """Rebuild a cache from ``state_dict()`` output (tensors may be on the CPU)."""
        device = torch.device(device) if device is not None else (
            sd["fp4"].device if sd["fp4"].is_cuda else torch.device("cuda", torch.cuda.current_device()))
        fp4 = sd["fp4"].to(device=device, dtype=torch.uint8).contiguous()
        sf = sd["sf"].to(device=device, dtype=torch.uint8).contiguous()
        n, k = fp4.shape[0], fp4.shape[1] * 2
        assert sf.numel() == n * k // 16, "scale buffer size does not match the packed data"
        with torch.cuda.device(device):
            h = _lib.fp4b_weight_cache_import(fp4.data_ptr(), sf.data_ptr(), n, k, _stream_ptr(device))
        if not h:
            raise RuntimeError(f"fp4b_weight_cache_import failed ({_last_error()})")
        g = float(sd.get("global_scale", 1.0))
        if g != 1.0 and _lib.fp4b_weight_cache_set_alpha(h, 1.0 / g) != 0:
            _lib.fp4_weight_cache_free(ctypes.c_void_p(h))
            raise RuntimeError(f"fp4b_weight_cache_set_alpha failed ({_last_error()})")
        bias = sd.get("bias")
        if bias is not None:
            bias = bias.to(device)
        return cls._from_handle(h, sd["N_orig"], sd["K_orig"], device, bias)

    def free(self):
        """Free the cached weight's device memory (later forwards raise)."""
        if getattr(self, "_handle", None) and _lib is not None:
            _lib.fp4_weight_cache_free(ctypes.c_void_p(self._handle))
            self._handle = None
        self._staging = None

    def __enter__(self):
        return self

    def __exit__(self, *args):
        self.free()

    def __del__(self):
        self.free()

    def __repr__(self):
        size_mb = (self.fp4_bytes + self.sf_bytes) / 2 ** 20
        state = "freed" if not self._handle else "active"
        return "FP4WeightCache([%d, %d], %.1f MB, %s)" % (self.N_orig, self.K_orig, size_mb, state)


def fp4_quantize(weight: torch.Tensor, bias: torch.Tensor = None, global_scale: bool = False) -> FP4WeightCache:
    """Build an FP4WeightCache for `weight` (and `bias`); see that class."""
    return FP4WeightCache(weight, bias, global_scale=global_scale)


def fp4_cached_matmul(
    A: torch.Tensor,
    cache: FP4WeightCache,
) -> torch.Tensor:
    """q(A) @ W^T with W stored in `cache` ([M, K] or [b, M, K] in, [.., N] out);
    the same call as cache.forward(A)."""
    return cache.forward(A)


def fp4_cached_linear(
    x: torch.Tensor,
    cache: FP4WeightCache,
) -> torch.Tensor:
    """F.linear(x, W, bias) with W (and its bias) stored in `cache`; x is [..., K],
    the result [..., N]."""
    return cache.forward(x)


# ----------------------------------------------------------------------------
# Lower-level helpers (additive; used by tests, benchmarks and fp4_gemm_dist)
# ----------------------------------------------------------------------------

def quantize_to_buffers(x: torch.Tensor, rows_pad: int = None, k_pad: int = None):
    """Quantize a 2-D BF16 CUDA tensor into new (fp4 [rows_pad, k_pad/2], sf) uint8 tensors (async)."""
    assert x.dim() == 2 and x.is_cuda and x.dtype == torch.bfloat16
    rows, cols = x.shape
    rows_pad = rows_pad or _pad_to_multiple(max(rows, 1), 128)
    k_pad = k_pad or _pad_to_multiple(max(cols, 1), 128)
    x, ld = _rows_view(x)
    fp4 = torch.empty(rows_pad, k_pad // 2, dtype=torch.uint8, device=x.device)
    sf = torch.empty(rows_pad * k_pad // 16, dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        rc = _lib.fp4b_quantize(x.data_ptr(), rows, cols, ld, fp4.data_ptr(), sf.data_ptr(), rows_pad, k_pad,
                                _stream_ptr(x.device))
    if rc != 0:
        raise RuntimeError(f"fp4b_quantize failed with error code {rc} ({_last_error()})")
    return fp4, sf


def gemm_prequantized(a_fp4, a_sf, m: int, b_fp4, b_sf, n: int, k_pad: int, bias=None, C=None,
                      alpha: float = 1.0, beta: float = 0.0, out=None):
    """D[m, n] from already-quantized operands (async; BF16 out)."""
    dev = a_fp4.device
    D = out if out is not None else torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    c_ptr, ldc = (C.data_ptr(), C.stride(0)) if C is not None else (None, 0)
    b_ptr = bias.data_ptr() if bias is not None else None
    with torch.cuda.device(dev):
        rc = _lib.fp4b_gemm_prequant(a_fp4.data_ptr(), a_sf.data_ptr(), m, a_fp4.shape[0], b_fp4.data_ptr(),
                                     b_sf.data_ptr(), n, b_fp4.shape[0], k_pad, c_ptr, ldc, D.data_ptr(),
                                     D.stride(0), b_ptr, float(alpha), float(beta), _stream_ptr(dev))
    if rc != 0:
        raise RuntimeError(f"fp4b_gemm_prequant failed with error code {rc} ({_last_error()})")
    return D


def gemm_tile_width(m: int, n: int, k: int, sms: int = 148) -> int:
    """Output columns per tile the GEMM's time model picks for M x N x K on a
    device with `sms` SMs (no device work): 128 / 192 / 256, or the two-MMA
    320 / 384, on CTA pairs at every M."""
    w = _lib.fp4b_gemm_tile_width(m, n, k, sms)
    if w < 0:
        raise ValueError(f"gemm_tile_width: {_last_error()}")
    return w


def mma_rate(n0: int = 256, n1: int = 0, sf_copies: bool = False, sfb_atoms: int = 0, stages: int = 8192,
             reps: int = 5) -> dict:
    """Measured tensor-pipe rate of the block-scaled MMA on the current device
    (fp4b_mma_rate; operands resident in shared memory, no loads): the best of
    `reps` CUDA-event-timed launches after one warm-up launch.  Returns
    {"tflops", "ms", "pairs"}.  The defaults measure the dense NVFP4 peak."""
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev)
    pairs = _i(0)
    best = None
    for rep in range(reps + 1):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        rc = _lib.fp4b_mma_rate(n0, n1, 1 if sf_copies else 0, sfb_atoms, stages, ctypes.byref(pairs),
                                stream.cuda_stream)
        stop.record(stream)
        if rc != 0:
            raise RuntimeError(f"fp4b_mma_rate failed with error code {rc} ({_last_error()})")
        stop.synchronize()
        ms = start.elapsed_time(stop)
        if rep > 0 and (best is None or ms < best):
            best = ms
    flops = pairs.value * stages * 4 * 2 * 256 * (n0 + n1) * 64
    return {"tflops": flops / (best * 1e-3) / 1e12, "ms": best, "pairs": pairs.value}


def device_error(clear: bool = True) -> int:
    """Non-zero if a kernel gave up on a bounded wait (synchronises the device)."""
    return _lib.fp4b_device_error(1 if clear else 0)


def ipc_handle(t: torch.Tensor):
    """(64-byte CUDA IPC handle of the allocation holding t, byte offset of t in it)."""
    buf = ctypes.create_string_buffer(64)
    off = ctypes.c_long(0)
    with torch.cuda.device(t.device):
        if _lib.fp4b_ipc_get_handle(t.data_ptr(), buf, ctypes.byref(off)) != 0:
            raise RuntimeError(f"fp4b_ipc_get_handle failed ({_last_error()})")
    return buf.raw, off.value


def ipc_open(handle: bytes, offset: int, device) -> int:
    """Map another process's allocation (see ipc_handle) into this one; returns the address of its tensor."""
    with torch.cuda.device(device):
        p = _lib.fp4b_ipc_open_handle(handle, offset)
    if not p:
        raise RuntimeError(f"fp4b_ipc_open_handle failed ({_last_error()})")
    return p


def ipc_close(ptr: int, offset: int, device):
    with torch.cuda.device(device):
        _lib.fp4b_ipc_close(ptr, offset)


def peer_barrier(my_flags: torch.Tensor, peer_flag_ptrs, peer_ranks, my_rank: int, epoch: int) -> None:
    """Queue fp4b_peer_barrier on the current stream of my_flags' device: signal
    `epoch` to every peer (their flag arrays, mapped at peer_flag_ptrs) and wait
    until every peer in peer_ranks has signalled it to this rank."""
    n = len(peer_flag_ptrs)
    ptrs = (_vp * n)(*peer_flag_ptrs)
    ranks = (_i * n)(*peer_ranks)
    with torch.cuda.device(my_flags.device):
        rc = _lib.fp4b_peer_barrier(my_flags.data_ptr(), ptrs, ranks, n, my_rank, epoch, _stream_ptr(my_flags.device))
    if rc != 0:
        raise RuntimeError(f"fp4b_peer_barrier failed with error code {rc} ({_last_error()})")


def copy2d(dst: int, dpitch: int, src: int, spitch: int, width_bytes: int, height: int, device) -> None:
    """Queue a strided device-to-device copy (fp4b_copy2d) on the current stream of `device`."""
    with torch.cuda.device(device):
        rc = _lib.fp4b_copy2d(dst, dpitch, src, spitch, width_bytes, height, _stream_ptr(device))
    if rc != 0:
        raise RuntimeError(f"fp4b_copy2d failed with error code {rc} ({_last_error()})")


def run_cached_into(x: torch.Tensor, cache: "FP4WeightCache", out: torch.Tensor) -> None:
    """x [M, K] @ cache^T (+ cache.bias, fused when BF16) written into `out` [M, cols], which may be a
    column slice of a wider buffer (unit column stride, any row stride).  Asynchronous."""
    x2, lda = _rows_view(x)
    m, k = x2.shape
    bias = cache.bias
    b_ptr = bias.reshape(-1).data_ptr() if (bias is not None and bias.is_cuda and bias.dtype == torch.bfloat16) else None
    if bias is not None and b_ptr is None:
        raise ValueError("run_cached_into fuses the bias: it must be a BF16 CUDA tensor")
    if out.dim() != 2 or out.stride(1) != 1 or out.shape[0] != m:
        raise ValueError("out must be a 2-D [M, cols] view with unit column stride")
    with torch.cuda.device(x2.device):
        rc = _lib.fp4b_run_cached_ex(x2.data_ptr(), m, k, lda, cache._handle, out.shape[1], None, 0, out.data_ptr(),
                                     out.stride(0), b_ptr, 1.0, 0.0, _stream_ptr(x2.device))
    if rc != 0:
        raise RuntimeError(f"fp4_gemm_run_cached failed with error code {rc} ({_last_error()})")


def run_cached_peers(x: torch.Tensor, cache: "FP4WeightCache", out: torch.Tensor, peer_ptrs) -> None:
    """This rank's columns of a column-parallel linear: x [M, K] @ cache^T (+ cache.bias, fused when BF16)
    into out [M, cols] (a column slice of a [M, N] buffer) and into the same columns of the peers'
    buffers (device addresses in peer_ptrs, already offset).  Asynchronous; order the ranks afterwards."""
    x2, lda = _rows_view(x)
    m, k = x2.shape
    bias = cache.bias
    b_ptr = bias.reshape(-1).data_ptr() if (bias is not None and bias.is_cuda and bias.dtype == torch.bfloat16) else None
    if bias is not None and b_ptr is None:
        raise ValueError("run_cached_peers fuses the bias: it must be a BF16 CUDA tensor")
    arr = (_vp * len(peer_ptrs))(*peer_ptrs)
    with torch.cuda.device(x2.device):
        rc = _lib.fp4b_run_cached_peers(x2.data_ptr(), m, k, lda, cache._handle, out.shape[1], out.data_ptr(),
                                        out.stride(0), arr, len(peer_ptrs), b_ptr, _stream_ptr(x2.device))
    if rc != 0:
        raise RuntimeError(f"fp4b_run_cached_peers failed with error code {rc} ({_last_error()})")
