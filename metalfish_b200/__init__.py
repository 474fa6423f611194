"""B200-native BT4 attention-body forward for the MetalFish NN backend path."""
from .synthetic import BT4, SMALL, TINY, CONFIGS, NetConfig, generate  # noqa: F401
