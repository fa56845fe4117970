"""CPU oracle for the optiz-qwen decode hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference algorithms that the CUDA path in
``optiz_qwen_b200`` replaces:

* ``kv_quant``  -- groupwise asymmetric uint4 quantisation and nibble packing
  (optiz_qwen/compression/qserve_kv_cache.py:313-372), plus the paged layout
  and page allocation policy used by the B200 cache.
* ``attention`` -- fp32 decode attention over the dequantised cache and the
  log-sum-exp merge of partial results.
* ``gdn``       -- the gated delta rule, token-by-token and chunked
  (transformers models/qwen3_5/modeling_qwen3_5.py:210-353, the functions the
  reference's GDN hook falls back to).

Parity is pinned by golden vectors produced by the reference's own code (see
``tests/golden/make_golden.py``); ``tests/test_oracle_golden.py`` checks this
package against them.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or the timed CPU baseline.  The product path
(``optiz_qwen_b200``) never imports it and never falls back to it.
"""
