"""CPU oracle for the SD1.5 UNet forward — TEST INFRASTRUCTURE ONLY.

This package is the checker, never the product. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it. The CUDA engine (``libsdg.so``) never calls into it, and the
product path has no CPU fallback.

Pinning: the ResNet-block and Transformer-block restatements reproduce the
reference's own PyTorch-generated golden vectors (``app/src/main/assets/rb``,
``app/src/main/assets/tf``) — see ``tests/test_oracle_kat.py``. The full-UNet
wiring (block order, skip LIFO, concat order) follows
``app/src/main/cpp/vk_engine.cpp:711-790``; no full-UNet golden output exists
in the reference checkout (the device self-test files ``IN_*``/``OUT_y`` named
at ``vk_engine.cpp:818`` are absent), so the whole-graph wiring is pinned only
through the two block KATs.
"""
