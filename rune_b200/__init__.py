"""rune_b200: B200-native energy / force / virial engine for RUNE's NEP4 and Möbius models.

Public API mirrors the reference packages:

* ``rune_b200.mobius.plugin`` — ``PLUGIN_NAME``, ``resolve_params``, ``build_model``,
  ``get_ddp_options``, ``load_model``, ``build_calculator`` (rune/mobius/plugin.py)
* ``rune_b200.nep.plugin`` — the same for NEP4 (rune/nep/plugin.py)
* ``rune_b200.runtime`` — the C-ABI binding (``include/rune_b200.h``) and the Engine handle.

All compute runs in the CUDA library ``rune_b200/_lib/librune_b200.so`` (sm_100a).
"""

__version__ = "0.1.0"
