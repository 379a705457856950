"""CPU oracle for the ``sparse_attn_sharedkv`` hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the algorithms of the reference repository
``yangqiang2018/dsv4_planB`` for the one path this project accelerates:

* ``golden_np``   -- numpy restatement of the fp32 golden attention model
  (``sparse_attn_sharedkv_tilelang/golden.py:28-204``) operating directly on
  the paged inputs of the public API, plus the index-resolution rule
  (``golden.py:28-66``) as a stand-alone function.
* ``sas_metadata_ref.c`` / ``metadata_ref`` -- plain-C restatement of the
  metadata tile scheduler (``sparse_attn_sharedkv_tilelang/metadata.py:258-1086``)
  and its ctypes wrapper.
* ``gen``         -- seeded input generators: a restatement of the reference's
  own generators (``golden.py:315-473``, ``test_sparse_attn_sharedkv.py:238-391``)
  and the generators for the BASELINE configurations.

Parity of this oracle with the reference is pinned by the fixtures under
``tests/golden/`` (made by ``tests/golden/make_fixtures.py``, which imports the
reference itself).  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` may import this package, and only as the checker
or the timed CPU baseline -- never as part of the product path.
"""
