"""Transcoders (behaviour of sae_lens/saes/transcoder.py; cases follow tests/saes/test_transcoder.py):
output width d_out, the skip path, JumpReLU thresholding and disk round trips for all four kinds."""

import pytest
import torch

from saelens_b200.models.sae import SAE
from saelens_b200.models.transcoder import (
    JumpReLUSkipTranscoder,
    JumpReLUSkipTranscoderConfig,
    JumpReLUTranscoder,
    JumpReLUTranscoderConfig,
    SkipTranscoder,
    SkipTranscoderConfig,
    Transcoder,
    TranscoderConfig,
)

KINDS = [(Transcoder, TranscoderConfig), (SkipTranscoder, SkipTranscoderConfig),
         (JumpReLUTranscoder, JumpReLUTranscoderConfig), (JumpReLUSkipTranscoder, JumpReLUSkipTranscoderConfig)]


def _make(cls, cfg_cls, seed=0):
    torch.manual_seed(seed)
    tc = cls(cfg_cls(d_in=12, d_sae=24, d_out=8, apply_b_dec_to_input=False))
    with torch.no_grad():
        for p in tc.parameters():
            p.copy_(torch.randn_like(p) * 0.3)
    return tc


@pytest.mark.parametrize("cls,cfg_cls", KINDS)
def test_forward_matches_formula(cls, cfg_cls):
    tc = _make(cls, cfg_cls)
    x = torch.randn(5, 12)
    with torch.no_grad():
        y = tc(x)
        pre = x @ tc.W_enc + tc.b_enc  # transcoders never subtract b_dec (it lives in the output space)
        f = torch.relu(pre) * (pre > tc.threshold) if hasattr(tc, "threshold") else torch.relu(pre)
        want = f @ tc.W_dec + tc.b_dec
        if hasattr(tc, "W_skip"):
            want = want + x @ tc.W_skip.T
    assert y.shape == (5, 8) and tc.d_out == 8
    torch.testing.assert_close(y, want, rtol=1e-5, atol=1e-5)
    out, feats = tc.forward_with_activations(x)
    torch.testing.assert_close(out, y)
    torch.testing.assert_close(feats, tc.encode(x))


@pytest.mark.parametrize("cls,cfg_cls", KINDS)
def test_disk_roundtrip(tmp_path, cls, cfg_cls):
    tc = _make(cls, cfg_cls, seed=1)
    tc.save_model(tmp_path)
    back = SAE.load_from_disk(tmp_path)
    assert type(back) is cls and back.cfg.d_out == 8
    x = torch.randn(4, 12)
    with torch.no_grad():
        torch.testing.assert_close(back(x), tc(x))


def test_transcoders_reject_b_dec_on_the_input():
    with pytest.raises(ValueError, match="apply_b_dec_to_input is not supported"):
        TranscoderConfig(d_in=12, d_sae=24, d_out=8, apply_b_dec_to_input=True)


def test_skip_transcoder_starts_with_a_zero_skip():
    tc = SkipTranscoder(SkipTranscoderConfig(d_in=12, d_sae=24, d_out=8, apply_b_dec_to_input=False))
    assert torch.count_nonzero(tc.W_skip) == 0 and tc.W_skip.shape == (8, 12)
