"""Tensor-level mirror of the reference's native module ``metal_liger_ext``.

The reference binds four Objective-C++/Metal functions through pybind
(csrc/bindings.mm:14-32, declared in csrc/metal_liger_ops.h:13-36):

    rms_norm_forward(x, weight, eps, kernel_dir)            -> [y, rms_cache]
    rms_norm_backward(x, weight, grad_out, eps, kernel_dir) -> [dx, dweight]
    swiglu_forward(gate, up, kernel_dir)                    -> out
    swiglu_backward(gate, up, grad_out, kernel_dir)         -> [dgate, dup]

The same four functions are provided here on CUDA tensors, calling the sm_100a
kernels through the C ABI.  ``kernel_dir`` is accepted and ignored (kernels are
compiled ahead of time, not from .metal sources at run time).
"""

from metal_liger_b200 import _torch_library as _tl


def rms_norm_forward(x, weight, eps, kernel_dir=""):
    y, rrms = _tl.rms_norm_forward_cuda(x, weight, eps, kernel_dir)
    return [y, rrms]


def rms_norm_backward(x, weight, grad_out, eps, kernel_dir=""):
    dx, dw = _tl.rms_norm_backward_cuda(x, weight, grad_out, eps, kernel_dir)
    return [dx, dw]


def swiglu_forward(gate, up, kernel_dir=""):
    return _tl.swiglu_forward_cuda(gate, up, kernel_dir)


def swiglu_backward(gate, up, grad_out, kernel_dir=""):
    dg, du = _tl.swiglu_backward_cuda(gate, up, grad_out, kernel_dir)
    return [dg, du]
