"""Token ids and sampling configuration of the native YuE2 protocol
(reference: src/protocol.rs:6-16 and 142-205)."""
import ctypes
from dataclasses import dataclass
from enum import IntEnum

from . import _lib

EOD = 151643
ABC_START = 151847
ABC_END = 151848
MUSIC_START = 151851
MUSIC_END = 151852
CODEC_OFFSET = 151853
CODEC_SIZE = 32768
LATENT_START = 184621
LATENT_END = 184622
LATENT_PAD = 184623
CONTEXT = 24576


class Phase(IntEnum):
    """sampling.rs:81-99; VOCAB is the vocabulary-generic variant (no window, no stop id)."""

    ABC = 0
    SEMANTIC = 1
    VOCAB = 2

    def end(self):
        return {Phase.ABC: ABC_END, Phase.SEMANTIC: MUSIC_END}.get(self)


@dataclass
class Sampling:
    """protocol.rs Sampling with its defaults (:153-165)."""

    temperature: float = 1.0
    top_p: float = 0.95
    top_k: int = 100
    repetition_penalty: float = 1.2
    penalty_window: int = 50
    min_tokens: int = 200
    max_tokens: int = 9000

    @classmethod
    def abc(cls):  # protocol.rs:167-177
        return cls(0.7, 0.9, 30, 1.005, 100, 32, 4096)

    def validate(self):  # protocol.rs:182-194
        import math
        t = self.temperature
        if (not math.isfinite(t) or not (0.0 <= t <= 5.0) or not math.isfinite(self.top_p) or self.top_p <= 0
                or self.top_p > 1 or self.top_k < 1 or not math.isfinite(self.repetition_penalty)
                or self.repetition_penalty <= 0 or not (1 <= self.penalty_window <= 100)
                or self.min_tokens > self.max_tokens or self.max_tokens < 1):
            raise ValueError("Invalid sampling configuration")
        return self

    def to_c(self):
        return _lib.CSampling(float(self.temperature), float(self.top_p), int(self.top_k),
                              float(self.repetition_penalty), int(self.penalty_window), int(self.min_tokens),
                              int(self.max_tokens))
