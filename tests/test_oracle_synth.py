"""The oracle's synthetic-layer generator (oracle/spt_synth.c) against the
CUDA library's host generator (spt_synth_layer_host): same bytes for every
tensor, so the CPU baseline and the reference arm of bench.py can build the
benchmark's weights without loading the library under test.  CPU only: the
library's host generator needs no GPU."""
import numpy as np
import pytest

from oracle import oracle


@pytest.mark.parametrize("seed,zipf,rbias,ebias", [(0, 0.0, True, True), (1, 0.0, True, True),
                                                    (2, 1.1, True, True), (3, 0.0, False, True),
                                                    (7, 0.0, True, False)])
def test_synth_layer_same_bytes(spt, seed, zipf, rbias, ebias):
    cfg = spt.Config(256, 192, 16, 4)
    kw = dict(seed=seed, zipf_s=zipf, zipf_beta=0.9 if zipf else 0.0, router_bias=rbias, expert_bias=ebias)
    for layer in (0, 3):
        want = spt.synth_layer_host(cfg, spt.SynthParams(**kw), layer)
        got = oracle.synth_layer(256, 192, 16, oracle.synth_params(**kw), layer, threads=3)
        for k in want:
            assert np.array_equal(np.asarray(got[k]).view(np.uint8), np.asarray(want[k]).view(np.uint8)), (k, layer)


def test_synth_gpt_oss_router_and_experts(spt):
    """GPT-OSS shapes at the Zipf-skewed prefill seed: every tensor of the
    1.7 GB layer."""
    cfg = spt.Config(2880, 2880, 128, 4)
    for seed, zipf in ((2, 1.1),):
        p = spt.SynthParams(seed=seed, zipf_s=zipf, zipf_beta=0.9 if zipf else 0.0)
        want = spt.synth_layer_host(cfg, p)
        got = oracle.synth_layer(2880, 2880, 128, oracle.synth_params(seed=seed, zipf_s=zipf,
                                                                       zipf_beta=0.9 if zipf else 0.0))
        for k in want:
            assert np.array_equal(got[k].view(np.uint8), want[k].view(np.uint8)), (k, seed)


def test_synth_activations_and_norm(spt):
    for seed, stream in ((1, 1000), (4, 1000), (2, 7919 + 1000)):
        assert np.array_equal(oracle.synth_normal(seed, stream, 5000).view(np.uint32),
                              spt.synth_normal_host(seed, stream, 5000).view(np.uint32))
    p = spt.SynthParams(seed=4)
    for layer in (0, 35):
        assert np.array_equal(oracle.synth_norm(4, layer, 2880).view(np.uint32),
                              spt.synth_norm_host(p, layer, 2880).view(np.uint32))
