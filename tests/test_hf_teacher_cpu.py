"""Cross-tokenizer distillation from a Hugging Face teacher on CPU (reference tests: tests/test_cross_tokenizer.py).
A tiny GPT-2 with its own byte-level BPE tokenizer is trained and saved offline; the teacher wrapper exposes
next-token probabilities with character end offsets, a character-level student distils from it with the exact
marginal loss (its cross-tokenizer loss falls), a BPE student runs the ULD loss, and conflicting or broken teacher
options are refused."""

import json

import pytest
import torch

from quantaweave_b200.data.pipeline import load_tokenizer
from quantaweave_b200.tools import cross_tokenizer as ct
from quantaweave_b200.tools.distill import build_parser, run_distillation
from quantaweave_b200.training.trainer import default_args, run_training

transformers = pytest.importorskip("transformers")
CPU = torch.device("cpu")
TEXTS = [f"story {i}: the quick brown fox jumps over the lazy dog." for i in range(60)]


@pytest.fixture(scope="module")
def setup(tmp_path_factory):
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers

    root = tmp_path_factory.mktemp("hf")
    data = root / "d.jsonl"
    data.write_text("".join(json.dumps({"text": t}) + "\n" for t in TEXTS))
    tok = Tokenizer(models.BPE(unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    tok.train_from_iterator(TEXTS, trainers.BpeTrainer(vocab_size=320, special_tokens=["<unk>", "<eos>"],
                                                       initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                                       show_progress=False))
    fast = transformers.PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="<unk>", eos_token="<eos>",
                                                pad_token="<eos>")
    torch.manual_seed(0)
    model = transformers.GPT2LMHeadModel(transformers.GPT2Config(vocab_size=len(fast), n_embd=48, n_layer=2,
                                                                 n_head=2, n_positions=128))
    batch = torch.tensor([fast.encode(t) + [fast.eos_token_id] for t in TEXTS[:8]])
    optimizer = torch.optim.AdamW(model.parameters(), lr=3e-3)
    for _ in range(80):  # enough for an informative next-token distribution on the template
        loss = model(input_ids=batch, labels=batch).loss
        optimizer.zero_grad()
        loss.backward()
        optimizer.step()
    teacher_dir = root / "teacher"
    model.save_pretrained(teacher_dir)
    fast.save_pretrained(teacher_dir)
    student = root / "student"
    run_training(default_args(data=[data], steps=6, batch_size=4, sequence_length=48, examples=60, hidden_size=32,
                              layers=1, ffn_size=32, attention_heads=2, total_experts=2, active_experts=1,
                              vocab_size=64, device="cpu", checkpoint_interval=0, no_power_tracking=True, lr=3e-3,
                              output=student, checkpoint_dir=root / "sck"))
    return root, data, teacher_dir, float(loss.detach()), student


def test_the_teacher_exposes_probabilities_end_offsets_and_token_strings(setup):
    _, _, teacher_dir, teacher_loss, _ = setup
    assert teacher_loss < 2.0
    teacher = ct.HFTeacher(str(teacher_dir), CPU)
    text = "story 3: the quick brown fox"
    probs, ends = teacher.next_token_probs(text)
    assert probs.shape == (len(ends), teacher.vocab_size) and ends[-1] == len(text) and ends == sorted(ends)
    assert torch.allclose(probs.sum(-1), torch.ones(len(ends)), atol=1e-4)
    strings = teacher.token_strings()
    ids = teacher.tokenizer(text, add_special_tokens=False)["input_ids"]
    assert len(strings) == teacher.vocab_size and "".join(strings[i] for i in ids) == text
    batch_probs, batch_ends = teacher.next_token_probs_batch([text, "the lazy dog"])
    assert torch.allclose(batch_probs[0], probs, atol=1e-5) and batch_ends[0] == ends  # padding changes nothing


def _args(tmp_path, student, data, teacher_dir, *extra):
    return build_parser().parse_args(["--student", str(student), "--teacher-data", str(data), "--hf-teacher",
                                      str(teacher_dir), "--output", str(tmp_path / "out"), "--checkpoint-dir",
                                      str(tmp_path / "ck"), "--sequence-length", "48", "--batch-size", "4",
                                      "--device", "cpu", "--checkpoint-interval", "0", "--no-archive", "--lr",
                                      "3e-3", "--examples", "60", *extra])


def test_a_character_student_distils_with_the_marginal_loss(setup, tmp_path, monkeypatch):
    _, data, teacher_dir, _, student = setup
    seen = []
    original = ct.CrossTokenizerLoss.__call__

    def spy(self, *args, **kwargs):
        loss, stats = original(self, *args, **kwargs)
        seen.append((float(loss.detach()), stats["aligned_fraction"], stats["mode"]))
        return loss, stats

    monkeypatch.setattr(ct.CrossTokenizerLoss, "__call__", spy)
    result = run_distillation(_args(tmp_path, student, data, teacher_dir, "--steps", "16", "--alpha", "1.0"))
    assert result["mode"] == "cross-tokenizer" and all(mode == "marginal" for *_, mode in seen)
    # a character position is trained where a teacher token ends there too: about one in four characters here
    assert all(0.1 < fraction < 1.0 for _, fraction, _ in seen)
    first, last = sum(v for v, *_ in seen[:4]) / 4, sum(v for v, *_ in seen[-4:]) / 4
    assert last < first, (first, last)


def test_a_bpe_student_runs_the_uld_loss(setup, tmp_path):
    root, data, teacher_dir, _, _ = setup
    bpe_student = tmp_path / "bpe_student"
    run_training(default_args(data=[data], steps=2, batch_size=4, sequence_length=24, examples=60, hidden_size=32,
                              layers=1, ffn_size=32, attention_heads=2, total_experts=2, active_experts=1,
                              vocab_size=300, tokenizer="bpe", tokenizer_path=tmp_path / "tok", device="cpu",
                              checkpoint_interval=0, no_power_tracking=True, output=bpe_student,
                              checkpoint_dir=tmp_path / "bck"))
    args = _args(tmp_path, bpe_student, data, teacher_dir, "--steps", "2")
    args.sequence_length = 24
    result = run_distillation(args)
    assert result["mode"] == "cross-tokenizer" and result["kl"] is not None and result["kl"] >= 0
    with pytest.raises(ValueError, match="marginal"):
        ct.CrossTokenizerLoss(ct.HFTeacher(str(teacher_dir), CPU), load_tokenizer(bpe_student), "marginal")


def test_conflicting_or_broken_teacher_options_are_refused(setup, tmp_path):
    _, data, teacher_dir, _, student = setup
    with pytest.raises(ValueError, match="one teacher"):
        run_distillation(_args(tmp_path, student, data, teacher_dir, "--teacher-checkpoint", str(student),
                               "--steps", "1"))
    with pytest.raises(Exception):
        run_distillation(_args(tmp_path, student, data, tmp_path / "no-such-teacher", "--steps", "1"))
    with pytest.raises(ValueError, match="cross-tokenizer loss"):
        ct.CrossTokenizerLoss(ct.HFTeacher(str(teacher_dir), CPU), load_tokenizer(student), "bogus")
