"""Host-side logic of the product against the oracle (CPU only): the batch
helpers (token ids, positions, next-token labels) and the AdamW hp rows."""
import numpy as np
import pytest

from oracle import oracle as O
from toy_b200.adamw import AdamW
from toy_b200.batch import next_token_labels, positions, synthetic_token_ids


@pytest.mark.parametrize("seed,n,vocab", [(5, 128, 512), (1000, 4096, 49152), (0, 7, 3), (-3, 33, 128256)])
def test_synthetic_ids_match_oracle_stream(seed, n, vocab):
    assert np.array_equal(synthetic_token_ids(seed, n, vocab), O.token_ids(seed, n, vocab))


@pytest.mark.parametrize("T,B", [(64, 1), (64, 4), (1, 3), (512, 8)])
def test_labels_and_positions(T, B):
    ids = O.token_ids(3, T * B, 512)
    ids[min(5, T * B - 1)] = 600          # out of vocabulary: no target
    assert np.array_equal(next_token_labels(ids, T, B, 512), O.next_token_labels(ids, T, B, 512))
    assert np.array_equal(positions(T, B), O.positions(T, B))


@pytest.mark.parametrize("step", [1, 2, 10, 1000])
def test_adamw_lora_hp(step):
    opt = AdamW.for_lora()
    opt.lr, opt.weight_decay = 1e-4, 0.01
    assert np.allclose(opt.hp(step), O.hp_lora(1e-4, step, wd=0.01), rtol=0, atol=0)


def test_adamw_mode_errors():
    with pytest.raises(ValueError):
        AdamW().hp(1)
    a = AdamW.for_lora()
    a.bias_correct = False
    with pytest.raises(ValueError):
        a.hp(1)
