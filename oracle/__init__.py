"""CPU oracle for the quantized MoE expert layer -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference's own CPU arithmetic for the MoE hot path:

* weight formats (dsv41/ref/kernel.py:10-29, 75-78, 91-98; dsv41/ref/fp4lib.c:12-30;
  dsv41/ckpt.py:5-6, 13, 41-50; dsv41/tt/weights.py:16-22),
* the router (dsv41/tt/moe.py:5-7, 15, 108-125),
* the SwiGLU expert FFN and the routed + shared combine (dsv41/tt/moe.py:133-142, 162, 180),
* the tensor-parallel split and all-reduce (dsv41/tt/moe.py:2-3; dsv41/tt/attn.py:19-21).

It is pinned against golden vectors produced by the reference's own ``kernel.py`` and its
``fp4lib.c`` (tests/golden/make_golden.py writes them; tests/test_oracle_golden.py checks them).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
package, and only as the checker or as the timed CPU baseline. The product path (the CUDA
library and its Python host code) never imports it and has no CPU fallback.
"""
