"""``mx.fast`` counterparts: fused primitives and the runtime kernel factory.

* ``rms_norm``  -> ``phew_rms_norm`` (replaces ``mx.fast.rms_norm``, phew
  ``emit/codegen.py:401-404``);
* ``layer_norm`` -> ``phew_layer_norm`` (``mx.fast.layer_norm``,
  ``emit/codegen.py:406-411``); ``rope`` -> ``phew_rope`` (``mx.fast.rope``,
  ``emit/codegen.py:413-419``);
* ``scaled_dot_product_attention`` -> the tcgen05 flash-attention kernel
  (replaces ``mx.fast.scaled_dot_product_attention``, ``emit/codegen.py:421-426``);
* ``cuda_kernel`` -> :class:`phew_b200.kernel.CudaKernel`, the analogue of
  ``mx.fast.metal_kernel`` (``ir/importer.py:55-94``) and of MLX's own
  ``mx.fast.cuda_kernel`` (listed in phew ``ir/op_registry.py:324-329``).
  Kernel objects are memoised by their definition, so the emitted code that
  constructs them inside the function body (``emit/codegen.py:488-495``)
  compiles once and reuses the object on every call.
"""

from __future__ import annotations

from ..kernel import CudaKernel

_kernels: dict[tuple, CudaKernel] = {}


def cuda_kernel(name, input_names, output_names, source, header="", ensure_row_contiguous=True,
                atomic_outputs=False, **_):
    key = (name, tuple(input_names), tuple(output_names), source, header,
           bool(ensure_row_contiguous), bool(atomic_outputs))
    k = _kernels.get(key)
    if k is None:
        k = CudaKernel(name, input_names, output_names, source, header,
                       ensure_row_contiguous=ensure_row_contiguous, atomic_outputs=atomic_outputs)
        _kernels[key] = k
    return k


def metal_kernel(name, input_names, output_names, source, header="", **_):
    raise NotImplementedError(
        "metal_kernel holds Metal Shading Language, which has no B200 path; emit CUDA C++ with "
        "phew_b200.emit.SubgraphCUDACodegen and build it with mx.fast.cuda_kernel"
    )


def rms_norm(x, weight=None, eps=1e-5, **_):
    from ..ops import rms_norm as _rms

    return _rms(x, weight, eps)


def layer_norm(x, weight=None, bias=None, eps=1e-5, **_):
    from ..ops import layer_norm as _ln

    return _ln(x, weight, bias, eps)


def rope(x, dims, *, traditional=False, base=10000.0, scale=1.0, offset=0, **_):
    from ..ops import rope as _rope

    return _rope(x, dims, traditional=traditional, base=base, scale=scale, offset=offset)


def quantized_scaled_dot_product_attention(q, k, v, scale_k, biases_k, scale_v, biases_v, *,
                                           scale=1.0, bits=4, group_size=64, mask=None, **_):
    from ..ops import quantized_sdpa

    return quantized_sdpa(q, k, v, scale_k, biases_k, scale_v, biases_v, scale=scale, bits=bits,
                          group_size=group_size, mask=mask)


def scaled_dot_product_attention(q, k, v, *, scale=1.0, mask=None, **_):
    from ..ops import scaled_dot_product_attention as _sdpa

    return _sdpa(q, k, v, scale=scale, mask=mask)
