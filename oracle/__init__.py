"""CPU oracle for the packed GGUF hot path -- TEST INFRASTRUCTURE ONLY.

A C restatement of the reference's Vx CPU kernels (packed_ref.c,
kernels_ref.c, fp8_ref.c) built into oracle/_build/ by oracle/Makefile.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import or load anything here; the product path (glm-vx_b200/) never does.
"""
