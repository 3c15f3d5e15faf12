"""Kernel entry points (ctypes over libpyrite_b200.so)."""
