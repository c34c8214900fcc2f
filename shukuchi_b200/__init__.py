"""B200 (sm_100a) decode path for the Shukuchi streaming LLM engine.

``libshk_cuda.so`` (built from ``csrc/``) holds every kernel and the C ABI of
``include/shk_cuda.h``; ``cuda.py`` is its ctypes mirror; ``engine/`` is the C
engine (GGUF reader, streaming loader, decode loop, CLI) over that ABI.
"""
