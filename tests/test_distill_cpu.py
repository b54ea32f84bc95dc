"""Distillation losses, cross-tokenizer alignment and the distillation CLI (reference tests:
tests/test_distill.py, tests/test_cross_tokenizer.py)."""

import torch
import torch.nn.functional as F

from quantaweave_b200.data.pipeline import CharTokenizer
from quantaweave_b200.tools.cross_tokenizer import (CrossTokenizerLoss, align_positions, first_char_matrix,
                                                    marginal_kl, uld_loss)
from quantaweave_b200.tools.distill import build_parser, distillation_loss, run_distillation


def test_distillation_loss_matches_batchmean_kl():
    torch.manual_seed(0)
    s, t = torch.randn(3, 9, 50), torch.randn(3, 9, 50)
    T = 2.0
    ref = F.kl_div(F.log_softmax(s[:, :-1].reshape(-1, 50) / T, -1), F.softmax(t[:, :-1].reshape(-1, 50) / T, -1),
                   reduction="batchmean") * T * T
    assert torch.allclose(distillation_loss(s, t, T, chunk_rows=5), ref, atol=1e-6)
    assert distillation_loss(s, s, T) < 1e-6


def test_align_positions_on_shared_boundaries():
    # student "ab|c|de" (lengths 2,1,2), teacher tokens end at 1, 3, 5 -> only offset 3 is shared (student token 1)
    assert align_positions([2, 1, 2], [1, 3, 5]) == [(1, 1)]
    # identical segmentation: every position but the last aligns
    assert align_positions([1, 1, 1], [1, 2, 3]) == [(0, 0), (1, 1)]
    # two teacher tokens end at the same offset: the later one wins
    assert align_positions([2, 1], [2, 2, 3]) == [(0, 1)]


class _CharTeacher:
    """A teacher whose tokens are single characters with a fixed next-token distribution."""

    def __init__(self, alphabet: str) -> None:
        self.alphabet = alphabet
        torch.manual_seed(1)
        self.table = torch.randn(len(alphabet)).softmax(-1)

    def token_strings(self):
        return list(self.alphabet)

    def next_token_probs(self, text):
        return self.table.expand(len(text), -1).clone(), list(range(1, len(text) + 1))


def test_marginal_loss_with_character_teacher():
    tok = CharTokenizer.build(["abcab"], 16)
    teacher = _CharTeacher("abc")
    loss_fn = CrossTokenizerLoss(teacher, tok, "auto")
    assert loss_fn.mode == "marginal"
    ids = torch.tensor([tok.encode("abcab")])
    logits = torch.randn(1, 5, 16, requires_grad=True)
    loss, stats = loss_fn(logits, ids)
    assert stats["aligned_positions"] == 4 and stats["aligned_fraction"] == 1.0
    matrix = first_char_matrix(teacher.token_strings(), tok, torch.device("cpu"), 16)
    ref = marginal_kl(logits[0, :4], teacher.table.expand(4, -1), matrix)
    assert torch.allclose(loss, ref)
    loss.backward()
    assert logits.grad[0, 4].abs().sum() == 0  # the last position has no successor


def test_uld_loss_is_permutation_invariant():
    p = torch.tensor([[0.7, 0.2, 0.1]])
    q = torch.tensor([[0.1, 0.7, 0.2, 0.0]])
    assert uld_loss(p, q) < 1e-7


def test_distillation_cli_logit_and_sequence_modes(tmp_path):
    from test_tools_cpu import _train

    data, _ = _train(tmp_path)
    common = ["--student", str(tmp_path / "out"), "--teacher-data", str(data), "--steps", "3",
              "--batch-size", "2", "--sequence-length", "32", "--examples", "40", "--device", "cpu",
              "--checkpoint-interval", "0", "--no-archive", "--lr", "1e-3"]
    logit = run_distillation(build_parser().parse_args(
        common + ["--teacher-checkpoint", str(tmp_path / "out"), "--output", str(tmp_path / "d1"),
                  "--checkpoint-dir", str(tmp_path / "c1")]))
    assert logit["mode"] == "logit" and logit["kl"] is not None and logit["kl"] < 0.5
    seq = run_distillation(build_parser().parse_args(
        common + ["--output", str(tmp_path / "d2"), "--checkpoint-dir", str(tmp_path / "c2")]))
    assert seq["mode"] == "sequence" and seq["kl"] is None
    assert (tmp_path / "d2" / "model.pt").exists()
