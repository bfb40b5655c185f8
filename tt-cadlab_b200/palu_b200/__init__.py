"""palu_b200: B200-native (sm_100a) Palu compressed-KV decode attention.

Host-side mirror of the reference's operator surface (ryankert01/tt-cadlab ``palu_tt``):

* ``palu_b200.fused``     -- table builders and ``palu_sdpa_decode`` (palu_tt/fused.py, the ttnn op surface)
* ``palu_b200.convert``   -- Palu dump reader and per-layer tensors (palu_tt/convert.py)
* ``palu_b200.attention`` -- ``PaluAttention`` decode layer with latent caches (palu_tt/attention.py)

The compute runs in ``libpalu_b200.so`` (C ABI: include/palu_b200.h), built by ``palu_b200.build``.
"""
__version__ = "0.1.0"
