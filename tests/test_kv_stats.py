"""KV-cache memory accounting of a generation: full-format bytes follow the committed length exactly; fp8 halves
the stored bytes, sliding windows cap them, KIVI codes old chunks, eviction counts only kept entries; the measured
allocation covers the cache buffers."""

import torch

import economize_b200 as eco
from economize_b200.models.config import tiny_llama
from economize_b200.models.llama import CausalLM, init_weights
from economize_b200.techniques.kv_evict import KVEvictConfig
from economize_b200.techniques.kv_quant import KIVIConfig, KVFp8Config


def _model(**kw):
    return init_weights(CausalLM(tiny_llama(num_layers=2, **kw), torch.float32, "cpu"), seed=0)


def _entry(m):  # bytes of one position's K and V in one layer, compute dtype
    c = m.config
    return 2 * c.num_kv_heads * c.head_dim * 4


def test_plain_row_bytes_follow_the_committed_length():
    m = _model()
    em = eco.apply(m)
    prompt = torch.arange(20) % 1000
    r = em.decode_batch([prompt], 6, decoding=eco.DecodeConfig(cycle_length=1))[0]
    kv = r.kv
    n = 20 + r.cycles  # every pass commits one token
    assert kv.passes == r.cycles
    assert kv.kv_bytes_full == 2 * n * _entry(m) and kv.kv_bytes == kv.kv_bytes_full
    assert kv.kv_bytes_read_full == sum(2 * (20 + i) * _entry(m) for i in range(kv.passes))


def test_fp8_window_and_kivi_are_modelled():
    m = _model()
    em = eco.apply(m, KVFp8Config(scale="none"))
    kv = em.decode_batch([torch.arange(30) % 900], 4, decoding=eco.DecodeConfig(cycle_length=1))[0].kv
    assert abs(kv.compression - 4.0) < 1e-9  # fp32 compute dtype vs one-byte codes
    w = _model(layer_types=("sliding_attention", "full_attention"), sliding_window=8)
    kvw = eco.apply(w).decode_batch([torch.arange(30) % 900], 4, decoding=eco.DecodeConfig(cycle_length=1))[0].kv
    n = 30 + 3
    assert kvw.kv_bytes == (8 + n) * _entry(w)
    k = eco.apply(_model(head_dim=128, num_heads=2, num_kv_heads=1, hidden_size=256), KIVIConfig(bits=2, residual=16))
    kvk = k.decode_batch([torch.arange(300) % 900], 3, decoding=eco.DecodeConfig(cycle_length=1))[0].kv
    assert kvk.compression > 1.5


def test_eviction_counts_kept_entries():
    m = _model()
    em = eco.apply(m, KVEvictConfig(method="streaming", budget=16, window=8, sink=4))
    kv = em.decode_batch([torch.arange(64) % 900], 3, decoding=eco.DecodeConfig(cycle_length=1))[0].kv
    assert kv.kv_bytes < kv.kv_bytes_full / 2
