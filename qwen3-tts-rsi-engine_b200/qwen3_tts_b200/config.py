"""Model geometry of the Qwen3-TTS decode path (talker, code predictor, codec).

Shapes follow the 1.7B CustomVoice model the reference serves: talker and
predictor are Qwen3-style decoders (RMSNorm eps 1e-6, per-head q/k RMSNorm,
rotate-half RoPE, GQA, SwiGLU); the codec is the 12.5 Hz tokenizer-v2 decoder
(16-codebook RVQ, 8-layer sliding-window transformer, transposed-conv
upsampling with SnakeBeta to 24 kHz, 1920 samples per frame).
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace


@dataclass(frozen=True)
class DecoderConfig:
    layers: int
    hidden: int
    q_heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    eps: float = 1e-6
    theta: float = 1_000_000.0

    @property
    def q_width(self) -> int:
        return self.q_heads * self.head_dim

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def qkv_width(self) -> int:
        return self.q_width + 2 * self.kv_width

    def weight_bytes(self, dtype_bytes: int = 2) -> int:
        """Bytes of the per-step streamed weights (layers + LM head)."""
        per_layer = self.hidden * self.qkv_width + self.q_width * self.hidden + 3 * self.hidden * self.ffn
        return (self.layers * per_layer + self.hidden * self.vocab) * dtype_bytes


@dataclass(frozen=True)
class TalkerConfig(DecoderConfig):
    """Talker: codec-token LM over 3072 ids; ids >= vocab-1024 are control tokens."""
    eos: int = 2150
    codebooks: int = 16


@dataclass(frozen=True)
class PredictorConfig(DecoderConfig):
    """Code predictor: 15 autoregressive residual codebooks per frame."""
    groups: int = 15
    talker_hidden: int = 2048


@dataclass(frozen=True)
class CodecConfig:
    """12.5 Hz incremental codec decoder (tokenizer-v2 geometry)."""
    codebooks: int = 16
    codebook_size: int = 2048
    codebook_dim: int = 512
    semantic_codebooks: int = 1
    latent: int = 1024
    hidden: int = 512
    layers: int = 8
    heads: int = 8
    head_dim: int = 64
    ffn: int = 1024
    window: int = 72
    eps: float = 1e-5
    theta: float = 10_000.0
    upsampling_ratios: tuple = (2, 2)
    upsample_rates: tuple = (8, 5, 4, 3)
    decoder_dim: int = 1536
    layer_scale: float = 0.01

    @property
    def samples_per_frame(self) -> int:
        total = 1
        for r in tuple(self.upsampling_ratios) + tuple(self.upsample_rates):
            total *= r
        return total


TALKER = TalkerConfig(layers=28, hidden=2048, q_heads=16, kv_heads=8, head_dim=128, ffn=6144, vocab=3072)
PREDICTOR = PredictorConfig(layers=5, hidden=1024, q_heads=16, kv_heads=8, head_dim=128, ffn=3072, vocab=2048)
CODEC = CodecConfig()


def tiny_talker(layers: int = 2) -> TalkerConfig:
    """Reduced talker for CPU-checkable parity (same head geometry)."""
    return replace(TALKER, layers=layers, hidden=256, ffn=512, vocab=3072)


def tiny_predictor(layers: int = 2) -> PredictorConfig:
    return replace(PREDICTOR, layers=layers, hidden=256, ffn=512, vocab=2048, talker_hidden=256)


@dataclass(frozen=True)
class PromptConfig:
    """CustomVoice prompt geometry (custom_voice_prompt.py:23-70).

    Text ids are embedded by a [text_vocab, text_hidden] table and mapped to the
    talker width by ``text_projection`` (fc1 text_hidden -> text_hidden with
    SiLU, fc2 -> hidden, both with bias). Codec-side control ids (think tags,
    language ids, speaker ids, codec pad/bos) index the talker's codec
    embedding; they all sit in the last 1024 ids the sampler masks out.
    The special text ids follow the Qwen chat template the reference tokenizes
    (role tokens first, five template tokens last).
    """
    text_vocab: int = 151936
    text_hidden: int = 2048
    hidden: int = 2048
    im_start: int = 151644
    im_end: int = 151645
    assistant: int = 77091
    user: int = 872
    newline: int = 198
    tts_pad: int = 151671
    tts_bos: int = 151672
    tts_eos: int = 151673
    codec_pad: int = 2148
    codec_bos: int = 2149
    codec_think: int = 2154
    codec_nothink: int = 2155
    codec_think_bos: int = 2156
    codec_think_eos: int = 2157
    languages: tuple = (("english", 2050), ("chinese", 2055), ("japanese", 2058), ("korean", 2064))
    speakers: tuple = (("voice_a", 3000), ("voice_b", 3001))
    dialects: tuple = ()   # (speaker, dialect-language) pairs; a dialect speaker's Chinese/auto
                           # prompts use the dialect's language id

    @property
    def language_ids(self) -> dict:
        return dict(self.languages)

    @property
    def speaker_ids(self) -> dict:
        return dict(self.speakers)


PROMPT = PromptConfig()


def tiny_prompt(hidden: int = 256) -> PromptConfig:
    """Reduced text vocabulary and width for CPU-checkable parity (special ids remapped)."""
    return replace(PROMPT, text_vocab=1024, text_hidden=hidden, hidden=hidden, im_start=1000, im_end=1001,
                   assistant=1002, user=1003, newline=1004, tts_pad=1005, tts_bos=1006, tts_eos=1007)
