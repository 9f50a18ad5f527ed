"""The encoder's convolutional front on this library's kernels (csrc/conv.cu).

Conv2d(kernel 3, stride 2, padding 1) + bias + GELU, as the audio tower's conv2d1-3 each
followed by F.gelu (models/audio_encoder.py:145-175): conv2d1 (one input channel) as a
direct stencil, conv2d2/conv2d3 as tcgen05 implicit GEMMs.

* Each convolution against a float64 convolution of the same bf16 inputs, rounded the
  way the reference rounds (bf16 convolution output, bias added and rounded, GELU
  rounded): at least 99.5 % of outputs bit-identical, every one within four bf16 steps
  of the largest of the output, its pre-GELU value and the convolution value (plus 2^-12).
  The chain rounds three times, so an fp32 sum that lands on the other side of a bf16
  boundary than the float64 one moves the output by a few steps; cuDNN's own fp32
  convolution (TF32 on, torch's default) differs from this float64 chain by the same
  0.03 at most and matches it on 99.8-99.9 % of outputs.
* The whole front (three convolutions + conv_out, as the engine runs it) against the
  fp32 oracle (oracle/model.py ``conv_front``, a restatement of modeling_qwen3_asr.py
  700-710) within the attention tolerance scaled to the output: max |err| <= 2e-2 and
  mean |err| <= 2e-3 of the largest output magnitude.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _ref_conv(x_nchw_bf16, w_bf16, b_bf16):
    """(output, pre-GELU value, convolution value), NCHW: the reference's rounding chain
    on a float64 convolution."""
    y = F.conv2d(x_nchw_bf16.double(), w_bf16.double(), None, stride=2, padding=1)
    yb = (y.bfloat16().double() + b_bf16.double()[None, :, None, None]).bfloat16()
    return F.gelu(yb.double()).bfloat16(), yb, y


def _close(got, want, pre, conv, what):
    g, w = got.double(), want.double()
    exact = (g == w).double().mean().item()
    mag = torch.maximum(torch.maximum(w.abs(), pre.double().abs()), conv.abs()).clamp_min(2.0 ** -100)
    bound = 4 * torch.exp2(torch.floor(torch.log2(mag)) - 7) + 2.0 ** -12
    assert exact >= 0.995 and torch.all((g - w).abs() <= bound), \
        (what, exact, (g - w).abs().max().item())


@pytest.mark.parametrize("n,h,w,cin,cout", [
    (3, 128, 100, 1, 480),    # conv2d1 of a 0.6B / 1.7B chunk
    (2, 64, 50, 480, 480),    # conv2d2
    (3, 32, 25, 480, 480),    # conv2d3
    (5, 13, 11, 1, 32),       # the tiny test preset, odd sizes
    (4, 7, 6, 32, 32),
    (1, 9, 9, 64, 128),
    # more tiles than SMs: each persistent CTA walks several tiles and reuses both
    # accumulators (channel tiles of 240, 128 and 32)
    (64, 64, 50, 480, 480),
    (96, 32, 25, 64, 256),
    (600, 16, 16, 32, 32),
])
def test_conv_matches_reference_rounding(n, h, w, cin, cout):
    from voiceagent_b200 import kernels as kx

    g = torch.Generator(device="cuda").manual_seed(n * 1000 + cin)
    x = torch.randn(n, cin, h, w, device="cuda", generator=g).bfloat16()
    wt = (torch.randn(cout, cin, 3, 3, device="cuda", generator=g) * (2.0 / (9 * cin)) ** 0.5).bfloat16()
    b = (torch.randn(cout, device="cuda", generator=g) * 0.1).bfloat16()
    packed = kx.conv_pack_weight(wt)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    x_cl = x.permute(0, 2, 3, 1).contiguous()
    got = kx.conv3x3s2_gelu(x_cl, packed, b, c_out=cout, error_flag=err)
    torch.cuda.synchronize()
    assert err.item() == 0
    want, pre, conv = (t.permute(0, 2, 3, 1) for t in _ref_conv(x, wt, b))
    _close(got, want, pre, conv, f"conv {n}x{h}x{w} {cin}->{cout}")
    # the transposed output order used for conv2d3: [n][ox][oy][c]
    got_t = kx.conv3x3s2_gelu(x_cl, packed, b, c_out=cout, out_order="nxyc")
    assert torch.equal(got_t.permute(0, 2, 1, 3), got)


def test_encoder_front_matches_oracle():
    """Three convolutions + conv_out of the 0.6B encoder on 6 random chunks (one short)
    through AudioEncoder._downsample, against the fp32 oracle front."""
    from oracle import model as M
    from voiceagent_b200.checkpoint import PRESETS
    from voiceagent_b200.config import AudioEncoderConfig
    from voiceagent_b200.qwen3_asr.audio_encoder import AudioEncoder

    cfg = PRESETS["0.6b"]
    c, d = cfg["audio"]["downsample_hidden_size"], cfg["audio"]["d_model"]
    gen = torch.Generator().manual_seed(4)
    shapes = {"conv2d1.weight": (c, 1, 3, 3), "conv2d2.weight": (c, c, 3, 3),
              "conv2d3.weight": (c, c, 3, 3), "conv_out.weight": (d, c * 16),
              "conv2d1.bias": (c,), "conv2d2.bias": (c,), "conv2d3.bias": (c,)}
    weights = {}
    for name, shape in shapes.items():  # N(0, 0.02) like the checkpoints, biases non-zero
        std = 0.05 if name.endswith(".bias") else 0.02
        weights["audio_tower." + name] = (torch.randn(shape, generator=gen) * std).bfloat16()
    enc = AudioEncoder(AudioEncoderConfig(**cfg["audio"])).to("cuda", torch.bfloat16)
    with torch.no_grad():
        for k, v in weights.items():
            name = k[len("audio_tower."):]
            mod, attr = name.rsplit(".", 1)
            getattr(enc.get_submodule(mod), attr).copy_(v.cuda())
    rng = np.random.default_rng(6)
    mel = rng.standard_normal((6, 128, 100)).astype(np.float32) * 0.5
    mel[5, :, 37:] = 0.0  # a short last chunk, zero-padded like the engine's
    mel_bf16 = torch.from_numpy(mel).bfloat16()
    enc.prepare_kernels()
    got = enc._downsample(mel_bf16.cuda(), 6).float().cpu()
    oracle = M.OracleThinker.__new__(M.OracleThinker)  # only the front's weights are needed
    oracle.w = {k: v.float() for k, v in weights.items()}
    want = oracle.conv_front(mel_bf16.float())
    assert got.shape == want.shape
    err = (got - want).abs()
    scale = want.abs().max().item()
    assert err.max().item() <= 2e-2 * scale and err.mean().item() <= 2e-3 * scale, \
        (err.max().item(), err.mean().item(), scale)
