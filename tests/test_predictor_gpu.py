"""Code-predictor chain (15 codebooks x decoder layers + sampling) against the CPU oracle."""
import numpy as np
import pytest
import torch

from oracle import decoder as OD
from oracle import elementwise as E
from oracle import sampling as S
from tests.golden.inputs import normal, uniform

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16


def setup(cuda, batch, **sampling):
    from qwen3_tts_b200.config import tiny_predictor
    from qwen3_tts_b200.predictor import PredictorStep
    from qwen3_tts_b200.weights import decoder_weights, pack_decoder
    cfg = tiny_predictor(layers=2)
    weights = decoder_weights(cfg, seed=21)
    talker_emb = torch.from_numpy(normal(22, (3072, cfg.talker_hidden), 0.02)).to(BF16)
    step = PredictorStep(cfg, pack_decoder(weights, cuda), talker_emb.to(cuda), batch, cuda, record_logits=True,
                         **sampling)
    step.capture()
    hidden = torch.from_numpy(normal(23, (batch, cfg.talker_hidden), 1.0)).to(BF16)
    first_codes = torch.from_numpy((uniform(24, (batch,)) * 2048).astype(np.int64))
    return cfg, weights, talker_emb, step, hidden, first_codes


def check_chain(cfg, weights, talker_emb, step, hidden, first_codes, draws_fn, top_p=1.0):
    codes = step.codes.cpu()
    gpu_logits = step.step_logits.cpu()
    first = talker_emb[first_codes].float()
    tables = OD.Tables(cfg.groups + 1, cfg.head_dim, cfg.theta)
    _, _, ref_logits = OD.predictor_frame(cfg, weights, hidden.float(), first, None, tables, mode="bf16f",
                                          uniforms_fn=draws_fn, forced_codes=codes[:, 1:], top_p=top_p)
    # per-step logits under teacher forcing: bf16-emulating oracle, same rounding points
    scale = ref_logits.abs().max()
    assert (gpu_logits - ref_logits).abs().max() <= 3e-2 * max(1.0, float(scale))
    # every code is the categorical draw of the GPU's own logits with that step's uniform
    flips = 0
    for s in range(cfg.groups):
        expect = S.categorical(gpu_logits[s], draws_fn(s), top_p=top_p)
        flips += int((expect[:, 0] != codes[:, s + 1]).sum())
    assert flips <= 1
    assert torch.equal(codes[:, 0], first_codes)
    embeds = step.embeds.cpu()
    ref = E.frame_embed(codes, talker_emb, weights["embeddings"], torch.zeros_like(embeds))
    assert torch.equal(embeds, ref)


def test_predictor_chain_with_uniform_tables(cuda):
    cfg, weights, talker_emb, step, hidden, first_codes = setup(cuda, 5)
    draws = torch.from_numpy(uniform(25, (5, 16)))
    step.run(hidden.to(cuda), first_codes.to(cuda), draws=draws.to(cuda))
    torch.cuda.synchronize()
    check_chain(cfg, weights, talker_emb, step, hidden, first_codes, lambda s: draws[:, s + 1])
    step.close()


def test_predictor_chain_philox_top_p(cuda):
    seed = 987654321
    cfg, weights, talker_emb, step, hidden, first_codes = setup(cuda, 6, philox_seed=seed, top_p=0.95)
    offsets = torch.arange(6, dtype=torch.long) * 1000 + 17
    step.run(hidden.to(cuda), first_codes.to(cuda), offsets=offsets.to(cuda))
    torch.cuda.synchronize()

    def draws_fn(s):
        return torch.from_numpy(S.philox_uniform(seed, (offsets + s).numpy()))

    check_chain(cfg, weights, talker_emb, step, hidden, first_codes, draws_fn, top_p=0.95)
    step.close()
