"""The end-to-end decoder (adaptiveimi_b200/model_e2e.py) on one GPU through
the IMI cache: decoding with the dense work of each layer captured as CUDA
graphs generates the same tokens, and the same hidden state within bf16
rounding, as eager decoding of the same model and prompt."""
import pytest
import torch

from adaptiveimi_b200.model_e2e import DecoderConfig, TPDecoder, generate

pytestmark = pytest.mark.gpu

CFG = DecoderConfig(layers=2, hidden=1024, q_heads=8, kv_heads=1, head_dim=128, intermediate=2048, vocab=4096)
PROMPT, NEW = 8192, 8
KMEANS = {"max_iters": 5}


def _run(graphs: bool):
    dev = torch.device("cuda", 0)
    m = TPDecoder(CFG, dev, seed=7, attention="imi", std=0.05)
    ids = torch.randint(0, CFG.vocab, (PROMPT,), generator=torch.Generator().manual_seed(11)).to(dev)
    m.make_cache(PROMPT, NEW, budget=0.1, parts=2, kmeans=KMEANS)
    r = generate(m, ids, NEW, graphs=graphs)
    return r["tokens"], m.last_hidden.float().cpu()


def test_graphed_decode_matches_eager():
    t_eager, h_eager = _run(False)
    t_graph, h_graph = _run(True)
    assert len(t_eager) == NEW
    assert t_graph == t_eager
    torch.testing.assert_close(h_graph, h_eager, rtol=2e-2, atol=2e-2)
