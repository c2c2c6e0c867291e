"""B200 device runtime (runtime.py) and the `vx-gpu` backend (backend.py)."""
