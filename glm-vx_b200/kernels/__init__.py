"""Reference-compatible kernel boundary (packed.py, backend.py) over libglmvx_cuda.so."""
