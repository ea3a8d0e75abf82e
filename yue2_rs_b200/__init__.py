"""B200-native YuE2 autoregressive decode (sm_100a kernels behind a C ABI).

The compute path is libyue2cuda.so (built by `python -m yue2_rs_b200.build`); this
package is its Python mirror of the reference's model.rs / sampling.rs entry points.
"""
from . import _lib
from ._lib import Yue2Error
from .model import Cache, Config, Model
from .protocol import (ABC_END, CODEC_OFFSET, CODEC_SIZE, CONTEXT, EOD, MUSIC_END, Phase, Sampling)
from .sampling import Generated, Generator, Request, Session, choose, generate, generate_batch

__all__ = [
    "Cache", "Config", "Model", "Phase", "Sampling", "Generator", "Generated", "Request", "Session", "choose",
    "generate", "generate_batch", "Yue2Error", "EOD", "ABC_END", "MUSIC_END", "CODEC_OFFSET", "CODEC_SIZE",
    "CONTEXT",
]


def cuda_available():
    """True when libyue2cuda finds a usable sm_100 device (yue2_metal_available's counterpart)."""
    return bool(_lib.lib().yue2_cuda_available())
