"""bf16 arithmetic for the Triton interpreter (golden-generation infrastructure only).

The interpreter (``triton/runtime/interpreter.py``, Triton 3.6) stores bf16 tensors as raw
uint16 bit patterns and hands those patterns straight to numpy: ``a - b`` subtracts the
integers, ``tl.dot`` multiplies them as integers, and the fp32 -> bf16 conversion rounds
half-up with no carry into the exponent. ``bf16_interp_probe.npz`` records the first of
these. So the interpreter cannot run the reference's kernels on bf16 inputs as they are.

``install()`` makes the interpreter's bf16 arithmetic follow IEEE semantics, the way a
GPU executes it: every bf16 operand is widened to fp32 (exact), the operation runs in
fp32, and a bf16 result is rounded to nearest-even once. For +, -, *, / and sqrt of bf16
operands this equals the correctly rounded bf16 result (fp32 carries more than
2 * 8 + 2 significand bits, so the double rounding is innocuous). ``tl.dot`` on bf16
operands accumulates in fp32, as ``tl.dot`` does on the GPU. ``tl.sum`` of a bf16 vector
accumulates in fp32 in numpy's order and rounds once, the rule the interpreter already
applies to fp16 vectors. Nothing changes for other dtypes, so the reference's kernels run
unmodified on the patched interpreter and every fp32 / fp16 fixture is unaffected.
"""
from __future__ import annotations

import numpy as np

_INSTALLED = False


def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    """Widen bf16 bit patterns (uint16) to fp32 values (exact)."""
    u = np.asarray(u16).astype(np.uint16).astype(np.uint32) << np.uint32(16)
    return u.view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to bf16 (nearest, ties to even) and return the uint16 patterns.
    NaN stays a quiet NaN with its sign; infinities and overflow to infinity follow IEEE."""
    f = np.asarray(x, dtype=np.float32)
    u = np.ascontiguousarray(f).view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    rounded = (u + np.uint32(0x7FFF) + lsb) >> np.uint32(16)
    qnan = (u >> np.uint32(16)) | np.uint32(0x0040)
    out = np.where(np.isnan(f), qnan, rounded)
    return out.astype(np.uint16)


_FLOAT_BINARY = {np.add, np.subtract, np.multiply, np.divide, np.fmod,
                 np.minimum, np.maximum}
_COMPARE = {np.less, np.less_equal, np.greater, np.greater_equal, np.equal, np.not_equal}


def install() -> None:
    """Patch the interpreter's builder and reduction so bf16 arithmetic is IEEE bf16."""
    global _INSTALLED
    if _INSTALLED:
        return
    import triton.language as tl
    from triton.runtime import interpreter as itp

    B = itp.InterpreterBuilder
    TH = itp.TensorHandle
    bf16 = tl.bfloat16

    def is_bf16(h) -> bool:
        return getattr(h, "dtype", None) is not None and h.dtype.scalar == bf16

    def widen(h):
        return bf16_bits_to_f32(h.data) if is_bf16(h) else h.data

    orig_binary = B.binary_op

    def binary_op(self, lhs, rhs, op):
        if not (is_bf16(lhs) or is_bf16(rhs)):
            return orig_binary(self, lhs, rhs, op)
        if op in _COMPARE:
            return TH(op(widen(lhs), widen(rhs)), lhs.dtype.scalar)
        if op in _FLOAT_BINARY:
            out = op(widen(lhs).astype(np.float32), widen(rhs).astype(np.float32))
            return TH(f32_to_bf16_bits(out), bf16)
        return orig_binary(self, lhs, rhs, op)  # bitwise ops act on the patterns

    orig_unary = B.unary_op

    def unary_op(self, arg, op):
        if not is_bf16(arg):
            return orig_unary(self, arg, op)
        out = op(widen(arg).astype(np.float32))
        return TH(f32_to_bf16_bits(out), bf16)

    orig_fma = B.create_fma

    def create_fma(self, x, y, z):
        if not (is_bf16(x) or is_bf16(y) or is_bf16(z)):
            return orig_fma(self, x, y, z)
        # exact product and sum in fp64, one rounding to fp32, one to bf16
        out = (widen(x).astype(np.float64) * widen(y).astype(np.float64)
               + widen(z).astype(np.float64)).astype(np.float32)
        return TH(f32_to_bf16_bits(out), bf16)

    orig_clamp = B.create_clampf

    def create_clampf(self, arg, lo, hi, propagate_nans):
        if not is_bf16(arg):
            return orig_clamp(self, arg, lo, hi, propagate_nans)
        out = np.clip(widen(arg), widen(lo), widen(hi))
        return TH(f32_to_bf16_bits(out), bf16)

    orig_dot = B.create_dot

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if not (is_bf16(a) or is_bf16(b)):
            return orig_dot(self, a, b, d, input_precision, max_num_imprecise_acc)
        acc = np.matmul(widen(a).astype(np.float32), widen(b).astype(np.float32),
                        dtype=np.float32)
        if is_bf16(d):
            return TH(f32_to_bf16_bits(acc + widen(d)), bf16)
        return TH((acc + d.data).astype(d.data.dtype), d.dtype.scalar)

    orig_cast = B.cast_impl

    def cast_impl(self, src, dst_type):
        s_bf, d_bf = is_bf16(src), dst_type.scalar == bf16
        if not (s_bf or d_bf):
            return orig_cast(self, src, dst_type)
        if s_bf and d_bf:
            return TH(src.data.copy(), bf16)
        if s_bf:
            f = bf16_bits_to_f32(src.data)
            return TH(f.astype(itp._get_np_dtype(dst_type)), dst_type.scalar)
        return TH(f32_to_bf16_bits(np.asarray(src.data).astype(np.float32)), bf16)

    orig_fp_to_fp = B.create_fp_to_fp

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        if is_bf16(src) or dst_type.scalar == bf16:
            return cast_impl(self, src, dst_type)
        return orig_fp_to_fp(self, src, dst_type, rounding_mode)

    B.binary_op = binary_op
    B.unary_op = unary_op
    B.create_fma = create_fma
    B.create_clampf = create_clampf
    B.create_dot = create_dot
    B.cast_impl = cast_impl  # the create_*_to_* casts call self.cast_impl
    B.create_fp_to_fp = create_fp_to_fp

    R = itp.ReduceOps
    orig_sum = R.sum

    def rsum(self, input):
        if input.dtype.scalar != bf16:
            return orig_sum(self, input)
        f = bf16_bits_to_f32(input.handle.data)
        s = np.sum(f, axis=self.axis, keepdims=self.keep_dims, dtype=np.float32)
        return self.to_tensor(f32_to_bf16_bits(s), input.dtype)

    orig_min_max = R.min_max

    def min_max(self, input, val_reduce_op, idx_reduce_op=None):
        x = input[0] if isinstance(input, tuple) else input
        if x.dtype.scalar != bf16:
            return orig_min_max(self, input, val_reduce_op, idx_reduce_op)
        f = bf16_bits_to_f32(x.handle.data)
        val = idx = None
        if val_reduce_op:
            val = self.to_tensor(f32_to_bf16_bits(val_reduce_op(f, axis=self.axis,
                                                                keepdims=self.keep_dims)), x.dtype)
        if idx_reduce_op:
            idx = self.to_tensor(idx_reduce_op(f, axis=self.axis, keepdims=self.keep_dims), tl.int32)
        if val is not None and idx is not None:
            return val, idx
        return val if val is not None else idx

    R.sum = rsum
    R.min_max = min_max
    _INSTALLED = True
