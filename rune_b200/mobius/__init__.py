"""Möbius (Local / MP / EQ) on the rune_b200 engine (mirrors rune/mobius)."""
