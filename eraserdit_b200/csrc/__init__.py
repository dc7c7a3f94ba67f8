"""CUDA sources of the C-ABI library and its build recipe (``build.py``)."""
