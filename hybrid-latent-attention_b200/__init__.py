"""B200-native (sm_100a) S6 hybrid latent-attention decode path.

Drop-in for ``hla/vllm_latent/s6_ops.py`` / ``s6_layer.py`` of Ch1nyzzz/hybrid-latent-attention:
``s6_ops`` mirrors the op API (backend ``'b200'``), ``s6_layer`` the per-(layer, loop) math,
``decode`` runs a whole Ouro-shaped decode step through the kernels.  The kernels live in
``libhla_s6.so`` (C ABI in ``include/hla_s6.h``), built in-tree by ``build.py``.

The directory name is not a Python identifier; import it with
``importlib.import_module('hybrid-latent-attention_b200')`` (or its ``.s6_ops`` etc.).
"""
PACKAGE = 'hybrid-latent-attention_b200'
