"""CPU oracle for the MojoLlama C-engine hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package, and only as the checker or the timed CPU baseline -- never as the thing
measured or shipped.  The product (``mojollama_b200``) never imports it and has
no CPU fallback.

Contents
  formats.py  numpy restatement of the GGUF block layouts the reference decodes
              (dequantize, quantize, our own K-quant encoders).
  ops.py      fp64/fp32 restatements of the per-op math (GEMV, RMSNorm, SiLU, RoPE,
              GQA, paged KV, MoE FFN, the reference's SSM decode step, ...).
  ref.py      ctypes loader for the reference C engine compiled from its own
              sources by ``oracle/Makefile`` into ``oracle/_ref/``.

Pinning: formats.py is checked bit-for-bit against gguf-py 0.19.0 (the
reference's un-pinned third-party dequantizer, ``Dockerfile:94`` of the
reference) through the committed fixtures in ``tests/golden/`` and, where the
reference C engine is built, against the reference's own ``*_dequantize_row``.
"""
