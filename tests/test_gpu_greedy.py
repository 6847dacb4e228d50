"""corm_greedy_embed (the greedy step between decode entries): the first
index of each row's maximum and that row of the embedding table, with ties at
several places in a row, rows at 16-byte-aligned and unaligned offsets (a
row stride that is not a multiple of 8) and a vocabulary that is not a
multiple of 8."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("vocab,ld", [(49152, 49152), (1003, 1011), (40, 40)], ids=["smollm2", "ragged", "small"])
def test_greedy_embed_first_argmax(vocab, ld):
    from cormorant_b200 import ops
    rng = np.random.default_rng(vocab)
    batch, dim = 7, 24
    lg = rng.integers(-3000, 3000, size=(batch, ld)).astype(np.int16)
    for b in range(batch):  # the row's maximum at several indices
        idx = rng.choice(vocab, size=1 + b % 4, replace=False)
        lg[b, idx] = 3000 + b
    table = rng.integers(-2**31, 2**31 - 1, size=(vocab, dim)).astype(np.int32)
    out = torch.zeros(batch * dim, dtype=torch.int32, device="cuda")
    ids = torch.full((batch,), -1, dtype=torch.int32, device="cuda")
    ops.greedy_embed(torch.from_numpy(lg.reshape(-1)).cuda(), torch.from_numpy(table.reshape(-1)).cuda(), out, ids,
                     batch=batch, vocab=vocab, dim=dim, ld=ld)
    want = np.argmax(lg[:, :vocab], axis=1)  # numpy returns the first index of a tie
    assert np.array_equal(ids.cpu().numpy(), want)
    assert np.array_equal(out.cpu().numpy().reshape(batch, dim), table[want])
