"""GPU parity of the greedy acceptance (srhpm_verify_accept, srhpm_argmax_shard + srhpm_accept_merge) against the
oracle's restatement of common_sampler_sample_and_accept_n with a greedy sampler and the reference's relaxed acceptance
(patch/srhpm.patch:9-35). The bar is identity: the emitted ids and their count."""
import numpy as np
import pytest
import torch

import oracle as O
import srhpm_b200 as S
from srhpm_b200 import _lib as L

pytestmark = pytest.mark.gpu

VOCAB = 151936  # the 27B-class target's vocabulary


def logits_with_winners(rng, rows, V, margin=0.5):
    lg = rng.standard_normal((rows, V)).astype(np.float32)
    win = rng.integers(0, V, rows)
    lg[np.arange(rows), win] = lg.max(axis=1) + margin
    return lg, win


def run(ctx, lg, draft, relax=0.0):
    ids, n = ctx.sample_and_accept_n(torch.from_numpy(lg).cuda(), torch.tensor(draft, dtype=torch.int32).cuda(), relax)
    torch.cuda.synchronize()
    ctx.check()
    return ids.cpu().numpy()[: int(n.item())].tolist()


@pytest.mark.parametrize("k", [0, 1, 2, 4, 8, 16])
def test_accept_all_prefixes(ctx, k):
    rng = np.random.default_rng(100 + k)
    lg, win = logits_with_winners(rng, k + 1, VOCAB)
    for stop in range(k + 1):  # first mismatch at `stop` (k: all accepted, bonus token emitted)
        draft = win[:k].copy()
        if stop < k:
            draft[stop] = (draft[stop] + 1 + rng.integers(0, VOCAB - 1)) % VOCAB
        got = run(ctx, lg, draft)
        assert got == O.accept(lg, draft), (k, stop)
        assert len(got) == (stop + 1 if stop < k else k + 1)


@pytest.mark.parametrize("relax", [0.05, 0.3, 2.0])
def test_accept_relaxed(ctx, relax):
    rng = np.random.default_rng(7)
    k = 8
    lg, win = logits_with_winners(rng, k + 1, VOCAB, margin=0.0)
    draft = win[:k].copy()
    for i in (2, 5):  # drafted tokens with logits just below the best
        alt = (win[i] + 17) % VOCAB
        lg[i, alt] = lg[i, win[i]] - (0.1 if i == 2 else 1.0)
        draft[i] = alt
    got = run(ctx, lg, draft, relax)
    assert got == O.accept(lg, draft, relax=relax)


def test_accept_ties_nan_and_small_vocab(ctx):
    rng = np.random.default_rng(8)
    V = 3001  # not a multiple of 4: the ragged tail path
    lg = rng.standard_normal((5, V)).astype(np.float32)
    lg[0, [10, 2000, 3000]] = 9.0        # tie: the first maximum
    lg[1, 0] = np.nan                    # a row starting with NaN: argmax 0 (sequential scan)
    lg[2, 17] = np.nan                   # NaN elsewhere: ignored
    lg[2, 1500] = 50.0
    lg[3, :] = -np.inf
    lg[3, 999] = -1e30
    draft = [10, 0, 1500, 999]
    got = run(ctx, lg, draft)
    assert got == O.accept(lg, draft)
    assert got == [10, 0, 1500, 999, int(np.argmax(lg[4]))]


def test_accept_strided_rows(ctx):
    rng = np.random.default_rng(9)
    big, win = logits_with_winners(rng, 5, VOCAB + 37)
    t = torch.from_numpy(big).cuda()[:, 5:5 + VOCAB]  # row stride VOCAB + 37, unaligned start
    lg = big[:, 5:5 + VOCAB].copy()
    draft = [int(np.argmax(lg[i])) for i in range(4)]
    ids, n = ctx.sample_and_accept_n(t, torch.tensor(draft, dtype=torch.int32).cuda())
    got = ids.cpu().numpy()[: int(n.item())].tolist()
    assert got == O.accept(lg, draft)


@pytest.mark.parametrize("n_shards", [2, 3, 8])
def test_accept_sharded_vocab(ctx, n_shards):
    rng = np.random.default_rng(10 + n_shards)
    k = 8
    lg, win = logits_with_winners(rng, k + 1, VOCAB)
    draft = win[:k].copy()
    draft[6] = (draft[6] + 5) % VOCAB
    lg[6, draft[6]] = lg[6, win[6]] - 0.2
    cuts = np.linspace(0, VOCAB, n_shards + 1).astype(int)
    cuts[1] += 3  # uneven shards
    t = torch.from_numpy(lg).cuda()
    d = torch.tensor(draft, dtype=torch.int32).cuda()
    recs = torch.stack([ctx.argmax_shard(t[:, cuts[s]:cuts[s + 1]], int(cuts[s]), d) for s in range(n_shards)])
    for relax in (0.0, 0.5):
        ids, n = ctx.accept_merge(recs, d, relax)
        got = ids.cpu().numpy()[: int(n.item())].tolist()
        assert got == O.accept(lg, draft, relax=relax) == run(ctx, lg, draft, relax)


def test_accept_repeat_and_status(ctx):
    rng = np.random.default_rng(11)
    lg, win = logits_with_winners(rng, 9, VOCAB)
    a = run(ctx, lg, win[:8])
    b = run(ctx, lg, win[:8])
    assert a == b == win.tolist()
    t = torch.from_numpy(lg).cuda()
    with pytest.raises(L.SrhpmError) as e:   # more drafted tokens than rows - 1
        ctx.sample_and_accept_n(t[:4], torch.tensor(win[:8], dtype=torch.int32).cuda())
    assert e.value.status == L.ERR_INVALID
    big = torch.zeros((18, 1000), dtype=torch.float32, device="cuda")
    with pytest.raises(L.SrhpmError) as e:   # 17 drafted tokens: beyond the verify path (ne[1] <= 16 + 1)
        ctx.sample_and_accept_n(big, torch.zeros(17, dtype=torch.int32, device="cuda"))
    assert e.value.status == L.UNSUPPORTED
