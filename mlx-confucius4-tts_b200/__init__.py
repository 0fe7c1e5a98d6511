"""c4s -- B200-native T2S sampling stage for Confucius4-TTS (host side)."""
from . import workloads  # noqa: F401
