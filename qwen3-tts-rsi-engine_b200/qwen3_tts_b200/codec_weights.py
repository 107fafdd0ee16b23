"""Seeded random-init codec decoder weights in the attribute layout ``pack_codec`` reads.

The real tokenizer-v2 decoder is a torch module tree (quantizer -> pre_conv ->
pre_transformer -> upsample -> decoder blocks); ``pack_codec`` only reads
parameters through attribute paths, so a tree of namespaces holding plain
tensors stands in for it when no checkpoint is available. Distributions:
matrices N(0, (0.5 / sqrt(fan_in))^2) so activations stay O(1); 1-D biases
N(0, 0.02); norm weights 1 + N(0, 0.02); layer scales and ConvNeXt gammas
0.1 + N(0, 0.02); SnakeBeta alpha = log U[0.5, 1.5], beta = N(0, 0.1);
codebook sums N(0, 1) with usage counts 0.5 + U[0, 1).
"""
from __future__ import annotations

import math
from types import SimpleNamespace as NS

import torch

from .config import CodecConfig


class _Draw:
    """Seeded draws; with ``seed=None`` every draw is an uninitialised tensor of the same shape
    (the tree a checkpoint is read into)."""

    def __init__(self, seed):
        self.g = None if seed is None else torch.Generator().manual_seed(seed)

    def randn(self, *shape):
        return torch.empty(shape) if self.g is None else torch.randn(shape, generator=self.g)

    def rand(self, *shape):
        return torch.empty(shape) if self.g is None else torch.rand(shape, generator=self.g)

    def matrix(self, *shape):
        fan_in = math.prod(shape[1:])
        return self.randn(*shape) * (0.5 / math.sqrt(fan_in))

    def bias(self, n):
        return self.randn(n) * 0.02

    def norm(self, n):
        return 1.0 + 0.02 * self.randn(n)

    def scale(self, n):
        return 0.1 + 0.02 * self.randn(n)

    def snake(self, channels):
        alpha = torch.log(0.5 + self.rand(channels))
        return NS(alpha=alpha, beta=self.randn(channels) * 0.1, no_div_by_zero=1e-9)

    def conv(self, c_in, c_out, k, dilation=1, groups=1):
        w = self.matrix(c_out, c_in // groups, k)
        return NS(conv=NS(weight=w, bias=self.bias(c_out), dilation=(dilation,), stride=(1,)),
                  padding=(k - 1) * dilation)

    def tconv(self, c_in, c_out, k, stride):
        w = self.randn(c_in, c_out, k) * (0.5 / math.sqrt(c_in))
        return NS(conv=NS(weight=w, bias=self.bias(c_out), stride=(stride,)), right_pad=k - stride)

    def linear(self, c_in, c_out, bias=True):
        return NS(weight=self.matrix(c_out, c_in), bias=self.bias(c_out) if bias else None)


def random_codec(cfg: CodecConfig, seed: int):
    return _codec_tree(cfg, _Draw(seed))


def codec_template(cfg: CodecConfig):
    """The codec tree with uninitialised tensors of the right shapes (filled from a checkpoint)."""
    return _codec_tree(cfg, _Draw(None))


def _codec_tree(cfg: CodecConfig, d: _Draw):

    def rvq(layers):
        books = [NS(_codebook=NS(embedding_sum=d.randn(cfg.codebook_size, cfg.codebook_dim),
                                 cluster_usage=0.5 + d.rand(cfg.codebook_size), epsilon=1e-5))
                 for _ in range(layers)]
        return NS(vq=NS(layers=books), output_proj=NS(weight=d.matrix(cfg.codebook_dim, cfg.codebook_dim, 1)))

    quantizer = NS(rvq_first=rvq(cfg.semantic_codebooks), rvq_rest=rvq(cfg.codebooks - cfg.semantic_codebooks),
                   n_q_semantic=cfg.semantic_codebooks)
    width = cfg.heads * cfg.head_dim
    layers = [NS(input_layernorm=NS(weight=d.norm(cfg.hidden)), q_proj=d.linear(cfg.hidden, width, False),
                 k_proj=d.linear(cfg.hidden, width, False), v_proj=d.linear(cfg.hidden, width, False),
                 o_proj=d.linear(width, cfg.hidden, False), attn_scale=d.scale(cfg.hidden),
                 post_attention_layernorm=NS(weight=d.norm(cfg.hidden)), gate_proj=d.linear(cfg.hidden, cfg.ffn, False),
                 up_proj=d.linear(cfg.hidden, cfg.ffn, False), down_proj=d.linear(cfg.ffn, cfg.hidden, False),
                 mlp_scale=d.scale(cfg.hidden)) for _ in range(cfg.layers)]
    transformer = NS(input_proj=d.linear(cfg.latent, cfg.hidden), layers=layers, norm=NS(weight=d.norm(cfg.hidden)),
                     output_proj=d.linear(cfg.hidden, cfg.latent))
    upsample = []
    for r in cfg.upsampling_ratios:
        block = NS(dwconv=d.conv(cfg.latent, cfg.latent, 7, groups=cfg.latent),
                   norm=NS(weight=d.norm(cfg.latent), bias=d.bias(cfg.latent), eps=1e-6),
                   pwconv1=d.linear(cfg.latent, 4 * cfg.latent), pwconv2=d.linear(4 * cfg.latent, cfg.latent),
                   gamma=d.scale(cfg.latent))
        upsample.append((d.tconv(cfg.latent, cfg.latent, r, r), block))
    mods = [d.conv(cfg.latent, cfg.decoder_dim, 7)]
    dim = cfg.decoder_dim
    for rate in cfg.upsample_rates:
        out = dim // 2
        units = [NS(act1=d.snake(out), conv1=d.conv(out, out, 7, dilation=dil), act2=d.snake(out),
                    conv2=d.conv(out, out, 1)) for dil in (1, 3, 9)]
        mods.append(NS(block=[d.snake(dim), d.tconv(dim, out, 2 * rate, rate)] + units))
        dim = out
    mods += [d.snake(dim), d.conv(dim, 1, 7)]
    return NS(cfg=cfg, quantizer=quantizer, pre_conv=d.conv(cfg.codebook_dim, cfg.latent, 3),
              pre_transformer=transformer, upsample=upsample, decoder=mods)
