"""B200-native (sm_100a) Summon-Verify Attention decode path."""

from . import kernels  # noqa: F401

__version__ = "0.1.0"
