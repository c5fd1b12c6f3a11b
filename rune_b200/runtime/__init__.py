"""Runtime layer: the C-ABI library binding, the build recipe and the Engine handle."""

from .library import RuneError, load_library  # noqa: F401
