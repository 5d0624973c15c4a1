"""ragrt_b200: a B200-native (sm_100a) implementation of RAGRT's plain-IVF `weft` search path."""
__version__ = "0.1.0"
