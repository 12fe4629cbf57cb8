"""B200-native (sm_100a) PECO attention hot path.

Drop-in for the reference's processor (``peco/processor.py``) and its ctypes
boundaries (``peco/clustering_cuda.py``, ``peco/attention_cuda.py``): the same
Python signatures over a C-ABI shared library, ``libpeco_b200.so``, built from
``peco_b200/csrc`` for sm_100a.  Submodules load the library lazily, so
importing the package never needs a GPU.
"""

__all__ = ["processor", "clustering", "quantization", "clustering_cuda", "attention_cuda", "synthetic"]
