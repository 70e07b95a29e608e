"""The MoE layer's top-k step (ffn_b200_topk, flash1017.rs:7280-7376) against the
oracle's router, through the C-ABI.

Up to 512 experts the step runs four warps per token (topk4_kernel), above that
one warp per token (topk_kernel); both are checked here.  Logits sit on a
1/64 grid, so distinct logits give scores far apart (no near-ties between the
GPU's and the CPU's expf) while equal logits give exact ties, which must go to
the lower expert index.  The partial planes are chosen so that their sum in
plane order is exact."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _grid_logits(rng, n_tok, n_exp, n_part):
    total = rng.integers(-256, 257, size=(n_tok, n_exp)).astype(np.float32) / 64.0
    planes = [rng.integers(-64, 65, size=(n_tok, n_exp)).astype(np.float32) / 64.0
              for _ in range(n_part - 1)]
    first = total - sum(planes) if planes else total
    return total, np.stack([first] + planes).astype(np.float32)


@pytest.mark.parametrize("n_exp", [384, 512, 640])
@pytest.mark.parametrize("top_k", [1, 6, 16])
@pytest.mark.parametrize("score_fn", [0, 1])
def test_topk_matches_oracle(ffn, cuda, oracle, n_exp, top_k, score_fn):
    import torch
    rng = np.random.default_rng(n_exp * 100 + top_k * 10 + score_fn)
    for n_tok, n_part in ((1, 1), (7, 3), (256, 3)):
        total, planes = _grid_logits(rng, n_tok, n_exp, n_part)
        idx, wt = ffn.topk(torch.from_numpy(planes).to(cuda), top_k, score_fn)
        torch.cuda.synchronize()
        ridx, rwt, _, _ = oracle.route(total, top_k, None, score_fn)
        np.testing.assert_array_equal(idx.cpu().numpy(), ridx)
        np.testing.assert_allclose(wt.cpu().numpy(), rwt, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("n_exp", [384, 640])
def test_topk_with_bias(ffn, cuda, oracle, n_exp):
    import torch
    rng = np.random.default_rng(7 + n_exp)
    total, planes = _grid_logits(rng, 64, n_exp, 2)
    bias = (rng.standard_normal(n_exp) * 0.05).astype(np.float32)
    idx, wt = ffn.topk(torch.from_numpy(planes).to(cuda), 6, 1, bias=torch.from_numpy(bias).to(cuda))
    torch.cuda.synchronize()
    ridx, rwt, _, _ = oracle.route(total, 6, bias, 1)
    ok = oracle.topk_agrees(idx.cpu().numpy(), ridx, oracle.biased_sorted(total, 6, bias, 1), tol=1e-6)
    assert ok.all()
    same = (idx.cpu().numpy() == ridx).all(axis=1)
    assert same.mean() > 0.95
    np.testing.assert_allclose(wt.cpu().numpy()[same], rwt[same], rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("n_exp", [384, 640])
def test_topk_nan_scores_are_never_selected(ffn, cuda, n_exp):
    """Token 0: every logit NaN -> six empty rounds (index 0x7fffffff, weight 0).
    Token 1: three finite logits -> those three in order, then empty rounds.
    Token 2: NaN everywhere but the last expert."""
    import torch
    lg = np.full((3, n_exp), np.nan, dtype=np.float32)
    lg[1, [5, 100, n_exp - 1]] = [0.5, 2.0, 1.0]
    lg[2, n_exp - 1] = -1.0
    idx, wt = ffn.topk(torch.from_numpy(lg).to(cuda), 6, 1)
    torch.cuda.synchronize()
    idx, wt = idx.cpu().numpy(), wt.cpu().numpy()
    none = 0x7FFFFFFF
    assert (idx[0] == none).all() and (wt[0] == 0).all()
    assert idx[1].tolist() == [100, n_exp - 1, 5, none, none, none]
    s = 1.0 / (1.0 + np.exp(-np.array([2.0, 1.0, 0.5])))
    np.testing.assert_allclose(wt[1, :3], s / s.sum(), rtol=1e-6)
    assert (wt[1, 3:] == 0).all()
    assert idx[2].tolist() == [n_exp - 1] + [none] * 5
    np.testing.assert_allclose(wt[2, 0], 1.0, rtol=1e-6)


def test_topk_rejects_bad_arguments(ffn, cuda):
    import torch
    lg = torch.zeros(4, 1, 8, device=cuda)
    with pytest.raises(ffn.FfnError):
        ffn.topk(lg, 6, 1)  # four planes: at most three
    with pytest.raises(ffn.FfnError):
        ffn.topk(torch.zeros(2, 8, device=cuda), 9, 1)  # top_k > n_exp
