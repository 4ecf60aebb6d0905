"""KernelSwift-B200: sm_100a kernels for KernelSwift's Sinkhorn, SparseAttention and
Indexer operators behind the reference's ``ModelNew`` interfaces.

Drop-in modules (same constructors, forwards, ``get_inputs`` and
``get_init_inputs`` as the reference's ``baseline/*.py``):
``kernelswift_b200/sinkhorn.py``, ``kernelswift_b200/sparse_attention.py``,
``kernelswift_b200/indexer.py``.  Torch-level ops: ``kernelswift_b200.ops``.
C ABI: ``include/ks_b200.h`` (``libks_b200.so``).
"""
__version__ = "0.1.0"
