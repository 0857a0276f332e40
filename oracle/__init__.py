"""CPU oracle for the packed-INT2 MLA content-cache path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package, and only as the checker or the timed CPU baseline.  The product package
(``mla_kv_quant_b200``) never imports it and has no CPU fallback.

What is restated here, and from where (paths are inside noforit/mla_kv_quant):

* ``codec``   -- the OSCAR Lloyd INT2 codec, ``mla_quant/oscar.py:120-144``,
  split into code extraction, 4-codes-per-byte packing and affine dequant, with
  the scalar handling of ``mla_quant/quantizer.py:31-35`` (HF path) and
  ``deployment/sglang/QuantKernel/mla_fused_writer.py:158-164`` (serving path).
* ``writer``  -- the fused decode writer's auxiliary stores (``k_pe``, the s4r16
  ring, the slot<->ring maps), ``mla_fused_writer.py:16-51``.
* ``decode``  -- absorbed MLA decode attention over the packed cache plus the BF16
  window rows, the math implied by ``deployment/patches/rolaq_sglang.patch:51-111,
  205-248`` and ``deployment/sglang/srt/mem_cache/rolaq_mla.py:56-71``.
* ``window``  -- the sink/recent token states of ``mla_quant/cache.py:775-800``.
* ``quantizer`` -- ``rotate_quantize`` (``mla_quant/quantizer.py:102-124``), the HF
  quantize-dequantize path, on the CPU; also the timed fallback of the CPU QDQ baseline.
* ``codec.encode_uniform`` -- OSCAR's uniform min/max INT2 baseline codec
  (``mla_quant/oscar.py:91-101``).

Parity status: the codec arithmetic is pinned against golden vectors produced by
importing the reference itself (``tests/golden/make_golden.py``).  The packed byte
order, the decode kernel and the ring lifecycle live in the un-vendored OSCAR fork
of SGLang (commit 19f85e13059de3da60686af4cbdd778b5671d9ff); for those the oracle
restates the semantics of the reference's call sites, and byte-level parity
against upstream is unpinned.
"""

from . import codec, writer, decode, window, quantizer  # noqa: F401
