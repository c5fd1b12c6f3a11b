"""NEP4 predictor on the rune_b200 engine (mirrors rune/nep)."""
