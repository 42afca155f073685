"""Drop-in for the reference's dense NVFP4 GEMM entry points
(kernels/gemm/submission.py:752 ``compile_kernel`` and :772 ``custom_kernel``).

``custom_kernel(data)`` takes the reference's 7-tuple, reads a, b and the two
permuted scale tensors, writes c in place on the current CUDA stream and
returns c, like the reference (submission.py:774-794).  The plain scale
tensors are ignored, as in the reference.
"""
from __future__ import annotations

import ctypes
import weakref

import torch

from . import _native
from .layout import SF_VEC, ceil_div, is_permuted_layout
from .task import gemm_input_t, gemm_output_t

_compiled = None
# Memo of validated argument sets: (weak refs to the 5 tensors, m, n, k, l).  A hit
# needs the very same tensor objects (still alive), so only an in-place change of
# their shape, strides or storage (resize_, set_, as_strided_) would bypass the
# checks.  Bounded, and holds no strong references.
_validated: dict = {}
_VALIDATED_MAX = 32
# output dtype of C -> the options' out_dtype
_OUT_DTYPES = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def compile_kernel():
    """Load the precompiled sm_100a library (the reference JIT-compiles here,
    submission.py:752-769).  Returns the callable entry point."""
    global _compiled
    if _compiled is None:
        _native.load()
        _compiled = custom_kernel
    return _compiled


def _check_operand(t: torch.Tensor, rows: int, kb: int, l: int, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if tuple(t.shape) != (rows, kb, l):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {(rows, kb, l)}")
    want = (kb, 1, rows * kb)
    if any(sz > 1 and st != w for sz, st, w in zip(t.shape, t.stride(), want)):
        raise ValueError(f"{name} must be K-major with batch outermost, strides {want}; got {t.stride()}")


def _current_stream(t: torch.Tensor) -> int:
    return torch._C._cuda_getCurrentRawStream(t.get_device())


def launch(a, b, sfa_perm, sfb_perm, c, m: int, n: int, k: int, l: int, stream=None,
           opt: _native.Nvfp4Options | None = None) -> None:
    """Raw launch on device pointers (tensors or ints); no layout checks."""
    lib = _native.load()
    ptr = lambda x: x if isinstance(x, int) else x.data_ptr()
    s = torch.cuda.current_stream().cuda_stream if stream is None else stream
    if opt is None:
        rc = lib.nvfp4_gemm(ptr(a), ptr(b), ptr(sfa_perm), ptr(sfb_perm), ptr(c), m, n, k, l, s)
    else:
        rc = lib.nvfp4_gemm_ex(ptr(a), ptr(b), ptr(sfa_perm), ptr(sfb_perm), ptr(c), m, n, k, l, s,
                               ctypes.byref(opt))
    _native.check(rc, "nvfp4_gemm")


def _validate(a, b, sfa_perm, sfb_perm, c):
    m, kb, l = a.shape
    n = b.shape[0]
    k = 2 * kb  # two e2m1 values per byte (submission.py:779)
    _check_operand(a, m, kb, l, "a")
    _check_operand(b, n, kb, l, "b")
    if c.dtype not in _OUT_DTYPES or tuple(c.shape) != (m, n, l):
        raise ValueError(f"c must be float16 (or bfloat16, float32) of shape {(m, n, l)}")
    if any(sz > 1 and st != w for sz, st, w in zip(c.shape, c.stride(), (n, 1, m * n))):
        raise ValueError(f"c must have strides {(n, 1, m * n)}; got {c.stride()}")
    sf_k = ceil_div(k, SF_VEC)
    if not is_permuted_layout(sfa_perm, m, sf_k, l) or not is_permuted_layout(sfb_perm, n, sf_k, l):
        raise ValueError("scale tensors must use the permuted (32, 4, rest_mn, 4, rest_k, l) layout")
    return m, n, k, l


def custom_kernel(data: gemm_input_t, opt: _native.Nvfp4Options | None = None) -> gemm_output_t:
    a, b, _, _, sfa_perm, sfb_perm, c = data
    key = (id(a), id(b), id(sfa_perm), id(sfb_perm), id(c))
    hit = _validated.get(key)
    if hit is not None and all(r() is t for r, t in zip(hit[0], (a, b, sfa_perm, sfb_perm, c))):
        m, n, k, l = hit[1]
    else:
        m, n, k, l = _validate(a, b, sfa_perm, sfb_perm, c)
        if len(_validated) >= _VALIDATED_MAX:
            _validated.clear()
        _validated[key] = (tuple(weakref.ref(t) for t in (a, b, sfa_perm, sfb_perm, c)), (m, n, k, l))
    lib = _native.load()
    want = _OUT_DTYPES[c.dtype]
    if opt is None and want:
        opt = _native.options(out_dtype=want)
    elif opt is not None and opt.out_dtype != want:
        raise ValueError(f"c is {c.dtype} but opt.out_dtype is {opt.out_dtype} (expected {want})")
    if opt is None:
        rc = lib.nvfp4_gemm(a.data_ptr(), b.data_ptr(), sfa_perm.data_ptr(), sfb_perm.data_ptr(),
                            c.data_ptr(), m, n, k, l, _current_stream(a))
    else:
        rc = lib.nvfp4_gemm_ex(a.data_ptr(), b.data_ptr(), sfa_perm.data_ptr(), sfb_perm.data_ptr(),
                               c.data_ptr(), m, n, k, l, _current_stream(a), ctypes.byref(opt))
    if rc:
        _native.check(rc, "nvfp4_gemm")
    return c


_ACTIVATIONS = {None: 0, "none": 0, "relu": 1, "gelu": 2}


def fused(data: gemm_input_t, bias: torch.Tensor | None = None, activation: str | None = None,
          opt: _native.Nvfp4Options | None = None) -> gemm_output_t:
    """``custom_kernel`` with a fused epilogue: C = act(A B^T + bias) in C's dtype.

    bias: None or an fp32 CUDA vector of N values (one per output column, shared by all
    batches); activation: None, "relu" or "gelu" (erf form); c may be float16, bfloat16 or
    float32.
    The bias and activation are applied to the fp32 accumulator before the rounding, as a
    cuBLASLt bias/relu epilogue does.
    """
    c = data[6]
    n = data[1].shape[0]
    if activation not in _ACTIVATIONS:
        raise ValueError(f"activation must be one of {sorted(k for k in _ACTIVATIONS if k)}")
    if bias is not None:
        if bias.dtype != torch.float32 or bias.numel() != n or not bias.is_cuda or not bias.is_contiguous():
            raise ValueError(f"bias must be a contiguous fp32 CUDA vector of {n} values")
    if opt is None:
        opt = _native.options()
    opt.bias = bias.data_ptr() if bias is not None else None
    opt.activation = _ACTIVATIONS[activation]
    opt.out_dtype = _OUT_DTYPES.get(c.dtype, 0)
    return custom_kernel(data, opt=opt)
