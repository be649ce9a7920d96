"""GPU: the tensor-core (tcgen05) GEMM that runs every projection of the chunked prefill and the batched decode
step, against fp64 matmuls of the reference-exact dequantized weights.

Precision: weights dequantized to fp16 (q * d rounded once, relative error <= 2^-11), activations fp16 with a
per-token power-of-two scale, fp32 accumulation in tensor memory -- max error within 4e-3 of the output's largest
magnitude.  Shapes follow BASELINE config 5 (N x K = 1536x1536, 256x1536, 8960x1536, 1536x8960, 151936x1536 at
M in {1, 8, 32, 128, 512} tokens) on the full-size model, and the small golden models' matrices (every weight format,
K not a multiple of 64, ragged token counts)."""

import numpy as np
import pytest
import torch

from oracle import vault_oracle as vo
from tests.golden.cases import CASES, case_config

pytestmark = pytest.mark.gpu
REL = 4e-3

_MODELS = {}


def engine(case_files, name):
    from vault_b200.model import VAULTv3ForCausalLM
    if name not in _MODELS:
        _MODELS[name] = VAULTv3ForCausalLM(case_files(name), device=0, max_sink=case_config(CASES[name]).max_sink)
    return _MODELS[name]


@pytest.mark.parametrize("name", ["mini_gqa_q8_0", "mini_gqa_q4_0", "mini_gqa_bf16", "tiny_seg_q8_0",
                                  "deep_hybrid_q4_0"])
@pytest.mark.parametrize("n_tok", [1, 5, 16, 77, 256, 300])
def test_gemm_matches_fp64(name, n_tok, case_files):
    m = engine(case_files, name)
    om = vo.OracleModel.from_file(case_files(name))
    g = torch.Generator().manual_seed(n_tok)
    li = 1
    for kind, key in ((2, "wq"), (4, "wk"), (8, "wo"), (12, "wd")):
        w = om.layers[li][key].astype(np.float64)
        x = torch.randn(n_tok, w.shape[1], generator=g)
        y = m.gemm(((li + 1) << 8) | kind, x, w.shape[0]).cpu().numpy().astype(np.float64)
        ref = x.numpy().astype(np.float64) @ w.T
        err = np.abs(y - ref).max() / (np.abs(ref).max() + 1e-12)
        assert err < REL, (key, err)
    # gate/up: the interleaved matrix comes back as [gate; up]
    gu = np.concatenate([om.layers[li]["wg"], om.layers[li]["wu"]]).astype(np.float64)
    x = torch.randn(n_tok, gu.shape[1], generator=g)
    y = m.gemm(((li + 1) << 8) | 10, x, gu.shape[0]).cpu().numpy().astype(np.float64)
    ref = x.numpy().astype(np.float64) @ gu.T
    assert np.abs(y - ref).max() / np.abs(ref).max() < REL


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_gemm_full_size_shapes(fmt):
    """BASELINE config 5 shapes on the full-size model (Hybrid Q4_0 keeps k/v and layers 0/1/26/27 q/o in Q8_0)."""
    from vault_b200 import synth
    from vault_b200.model import VAULTv3ForCausalLM
    m = VAULTv3ForCausalLM(synth.full_model_file(fmt, seed=0, n_sink=0), device=0, verify_crc=False)
    g = torch.Generator(device="cuda:0").manual_seed(7)
    li = 5
    for tid, rows, cols in (((li + 1) << 8 | 2, 1536, 1536), ((li + 1) << 8 | 4, 256, 1536),
                            ((li + 1) << 8 | 10, 17920, 1536), ((li + 1) << 8 | 12, 1536, 8960), (1, 151936, 1536)):
        w = m.dequant(tid, rows, cols).double()
        for n_tok in (1, 8, 32, 128, 512):
            x = torch.randn(n_tok, cols, generator=g, device="cuda:0")
            y = m.gemm(tid, x, rows).double()
            ref = x.double() @ w.T
            err = float((y - ref).abs().max() / ref.abs().max())
            assert err < REL, (tid, n_tok, err)
        del w
