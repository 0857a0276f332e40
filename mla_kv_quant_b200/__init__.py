"""B200 (sm_100a) packed-INT2 MLA content-cache path of RoLaQ (noforit/mla_kv_quant).

Host modules mirror the reference interfaces; the arithmetic runs in
``_lib/librolaq_b200.so`` (C ABI: ``include/rolaq_b200.h``):

* ``quantizer``         -- ``LearnedRotationQuantizer``, ``rotate_quantize`` (mla_quant API)
* ``rolaq_mla``         -- ``load_manifest``, ``load_layer_quantizers``, ``fold_read_rotation``
* ``mla_fused_writer``  -- ``try_fast_decode_store`` (serving writer plugin)
* ``mla_latent_int2``   -- ``scatter_pack_rows`` (general writer)
* ``mla_packed_decode`` -- ``packed_mla_decode_gf_fwd``, ``prepare_gf_splits`` (reader)
* ``pool``              -- ``PackedLatentPool`` (cache buffers and accounting)
* ``seqsplit``          -- sequence-split decode across ranks (NCCL all-gather + LSE merge)
"""

__version__ = "1.0.0"
