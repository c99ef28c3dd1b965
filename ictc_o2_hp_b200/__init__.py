"""B200-native ICTC-O2 tensor products: drop-in modules over hand-written sm_100a kernels.

Public names mirror the reference package ``ictc_o2_hp`` (src/ictc_o2_hp/__init__.py):
``TensorProduct``, ``TupleTensorProduct``, ``ComponentMajorTensorProduct``,
``UvuTensorProduct`` and ``RadialUvuTensorProduct``.  Imports are lazy so that the
package imports without a GPU.
"""

__version__ = "0.1.0"
__all__ = [
    "TensorProduct", "TupleTensorProduct", "ComponentMajorTensorProduct",
    "UvuTensorProduct", "RadialUvuTensorProduct", "__version__",
]


def __getattr__(name):
    if name in {"TensorProduct", "TupleTensorProduct", "ComponentMajorTensorProduct"}:
        from . import tensor_product
        return getattr(tensor_product, name)
    if name == "UvuTensorProduct":
        from .uvu import UvuTensorProduct
        return UvuTensorProduct
    if name == "RadialUvuTensorProduct":
        from .radial import RadialUvuTensorProduct
        return RadialUvuTensorProduct
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
