"""Test infrastructure: CPU oracles for the attention hot path.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
import this package, and only as the checker (or the timed CPU reference arm).
The product path (``fastflashattention_b200``) never imports it.

* ``flash_oracle``  numpy restatement of the reference Triton algorithm
  (``fastflash_attention/_kernel.py``), bf16 rounding where the reference casts.
* ``sdpa_oracle``   fp32 ``F.scaled_dot_product_attention`` (math backend) forward and
  autograd backward: the oracle of the reference's own tests
  (``tests/test_parity.py:32-35``).

Parity of ``flash_oracle`` is pinned against golden vectors produced by
``sdpa_oracle`` (``tests/golden/make_golden.py``) at the reference test gates.
"""
