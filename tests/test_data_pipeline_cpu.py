"""Data pipeline (reference tests: tests/test_data_pipeline.py, parts of tests/test_training_features.py):
tokenizers, per-domain corpora and windows, the stratified train/val split, token bins, curriculum, domain mixtures
and the deterministic, rank-partitioned batch stream."""

import json

import pytest
import torch

from quantaweave_b200.data.pipeline import (BatchStream, BPETokenizer, CharTokenizer, CurriculumConfig, DomainMixture,
                                            SentencePieceTokenizer, WindowDataset, build_corpus, difficulty_scores,
                                            load_token_bin, load_tokenizer, parse_domain_weights, read_rows,
                                            token_classes, write_token_bin)
from quantaweave_b200.utils.pii_redact import PIIRedactor


def _jsonl(path, rows):
    path.write_text("".join(json.dumps(r) + "\n" for r in rows))
    return path


@pytest.fixture
def two_domains(tmp_path):
    a = _jsonl(tmp_path / "prose.jsonl", [{"text": "the quick brown fox jumps over the lazy dog " * 6}] * 6)
    b = _jsonl(tmp_path / "code.jsonl", [{"text": "def f(x): return x + 1 # " * 6}] * 4)
    return [a, b]


def test_char_tokenizer_roundtrip_save_load_and_token_classes(tmp_path):
    tok = CharTokenizer.build(["hello world 123!"], 64)
    ids = tok.encode("hello 1!")
    assert tok.decode(ids) == "hello 1!"
    assert tok.encode("~")[0] == tok.unk_id  # unseen character
    tok.save(tmp_path)
    again = load_tokenizer(tmp_path)
    assert again.vocab == tok.vocab
    classes, names = token_classes(tok)
    assert classes.shape == (tok.vocab_size,)
    label = lambda ch: names[int(classes[tok.vocab[ch]])]  # noqa: E731
    assert (label("h"), label("1"), label(" "), label("!")) == ("letter", "digit", "space", "punct")
    assert names[int(classes[tok.eos_id])] == names[int(classes[tok.unk_id])] == "special"


def test_bpe_and_sentencepiece_train_save_and_roundtrip(tmp_path):
    texts = ["the cat sat on the mat", "the dog sat on the log", "a cat and a dog"] * 20
    for cls, name, size in ((BPETokenizer, "bpe", 300), (SentencePieceTokenizer, "sp", 40)):
        tok = cls.train(texts, size)
        ids = tok.encode("the cat sat")
        assert ids and tok.decode(ids).replace(" ", "") == "thecatsat"
        out = tmp_path / name
        tok.save(out)
        again = load_tokenizer(out)
        assert again.encode("the cat sat") == ids
    with pytest.raises(ValueError):
        SentencePieceTokenizer.train(texts, 40, algorithm="nope")


def test_domains_windows_split_and_token_bin(two_domains, tmp_path):
    rows = list(read_rows(two_domains))
    assert {d for d, _ in rows} == {"prose", "code"}
    tok = CharTokenizer.build((t for _, t in rows), 128)
    corpus = build_corpus(two_domains, tok)
    ds = WindowDataset(corpus, 15)
    assert len(ds) > 0 and ds.domains == ["prose", "code"]
    for i in range(len(ds)):  # windows never cross a domain boundary
        seg = corpus.segments[int(ds.window_domains[i])]
        start = int(ds.starts[i])
        assert seg.start <= start and start + 16 <= seg.start + seg.length
    train, val = ds.split_train_val(0.25, seed=3)
    t_starts, v_starts = set(train.starts.tolist()), set(val.starts.tolist())
    assert not (t_starts & v_starts) and t_starts | v_starts == set(ds.starts.tolist())
    assert set(val.window_domains.tolist()) == {0, 1}  # every domain is held out proportionally
    again_train, _ = ds.split_train_val(0.25, seed=3)
    assert torch.equal(again_train.starts, train.starts)
    other_train, _ = ds.split_train_val(0.25, seed=4)
    assert not torch.equal(other_train.starts, train.starts)
    with pytest.raises(ValueError):
        ds.split_train_val(1.5)
    meta = write_token_bin(two_domains, tok, tmp_path / "bin")
    assert meta
    mem, _ = load_token_bin(tmp_path / "bin")
    mem_ds = WindowDataset(mem, 15)
    assert len(mem_ds) == len(ds) and torch.equal(mem_ds.batch(range(len(ds))), ds.batch(range(len(ds))))


def test_batch_stream_is_deterministic_and_ranks_partition_the_global_batch(two_domains):
    tok = CharTokenizer.build((t for _, t in read_rows(two_domains)), 128)
    ds = WindowDataset(build_corpus(two_domains, tok), 15)
    whole = BatchStream(ds, 4, seed=9, world_size=1)
    ranks = [BatchStream(ds, 2, seed=9, rank=r, world_size=2) for r in range(2)]
    for step in (0, 5):
        a, da = whole.batch(step)
        assert torch.equal(a, whole.batch(step)[0])
        parts = [r.batch(step) for r in ranks]
        assert torch.equal(torch.cat([p[0] for p in parts]), a) and torch.equal(torch.cat([p[1] for p in parts]), da)
    assert not torch.equal(whole.batch(0)[0], whole.batch(1)[0])
    state = whole.state(3)
    assert state["samples_consumed"] == 12 and set(state["domain_weights"]) == {"prose", "code"}


def test_curriculum_starts_easy_and_widens_and_domain_mixture_blends(two_domains):
    tok = CharTokenizer.build((t for _, t in read_rows(two_domains)), 128)
    ds = WindowDataset(build_corpus(two_domains, tok), 15)
    scores = difficulty_scores(ds, "rarity", tok.vocab_size)
    assert scores.shape == (len(ds),)
    with pytest.raises(ValueError):
        difficulty_scores(ds, "nope", tok.vocab_size)
    cur = CurriculumConfig("rarity", start_fraction=0.25, steps=100)
    assert cur.fraction(0) == 0.25 and cur.fraction(100) == 1.0 and cur.stage(0) == 1 and cur.stage(100) == 4
    stream = BatchStream(ds, 64, seed=1, scores=scores, curriculum=cur)
    easy = set()
    for pool in stream.pools:  # step 0 may only draw from the easiest quarter of each domain
        reach = max(1, -(-pool.numel() // 4))
        easy |= {tuple(ds[int(i)].tolist()) for i in pool[:reach]}
    rows, _ = stream.batch(0)
    assert all(tuple(r.tolist()) in easy for r in rows)
    late, _ = stream.batch(100)
    assert any(tuple(r.tolist()) not in easy for r in late)
    mix = DomainMixture(["prose", "code"], {"prose": 1, "code": 0}, {"prose": 0, "code": 1}, steps=10)
    assert torch.allclose(mix.weights(0), torch.tensor([1.0, 0.0], dtype=torch.double))
    assert torch.allclose(mix.weights(5), torch.tensor([0.5, 0.5], dtype=torch.double))
    assert parse_domain_weights("prose=2, code=1") == {"prose": 2.0, "code": 1.0}
    with pytest.raises(ValueError):
        DomainMixture(["prose", "code"], {"prose": 1})
    mixed = BatchStream(ds, 32, seed=2, mixture=DomainMixture(["prose", "code"], {"prose": 0, "code": 1}))
    assert set(mixed.batch(0)[1].tolist()) == {1}


def test_pii_redaction_in_rows(tmp_path):
    path = _jsonl(tmp_path / "p.jsonl", [{"text": "mail me at jane.doe@example.com or call 555-123-4567"},
                                         {"text": "nothing to see here"}])
    redactor = PIIRedactor()
    rows = [t for _, t in read_rows([path], redactor=redactor)]
    assert "jane.doe@example.com" not in rows[0] and "555-123-4567" not in rows[0]
    assert rows[1] == "nothing to see here"
    assert sum(redactor.report().values()) >= 2
    assert [t for _, t in read_rows([path])][0].startswith("mail me at jane.doe")


def test_a_vocabulary_without_tokenizer_metadata_loads_as_characters(tmp_path):
    tok = CharTokenizer.build(["hello world"], 32)
    (tmp_path / "vocab.json").write_text(json.dumps(tok.vocab))  # an older checkpoint: no tokenizer_meta.json
    again = load_tokenizer(tmp_path)
    assert isinstance(again, CharTokenizer) and again.vocab == tok.vocab


def test_windows_stay_inside_one_domain_and_drop_partial_tails(tmp_path):
    data = _jsonl(tmp_path / "d.jsonl", [{"text": "aaaa", "domain": "x"}, {"text": "bbbbbbbbb", "domain": "y"},
                                          {"text": "aa", "domain": "x"}])
    tok = CharTokenizer.build(["ab"], 8)
    ds = WindowDataset(build_corpus([data], tok), 3)  # windows of 4 tokens
    a, b, eos = tok.vocab["a"], tok.vocab["b"], tok.eos_id
    # x: a a a a <eos> a a <eos> (8 tokens, 2 windows); y: 9 b's and <eos> (10 tokens, 2 windows, 2 left over)
    assert ds.domains == ["x", "y"] and ds.window_domains.tolist() == [0, 0, 1, 1]
    assert ds[0].tolist() == [a] * 4 and ds[1].tolist() == [eos, a, a, eos] and ds[2].tolist() == [b] * 4
    one = _jsonl(tmp_path / "stories.jsonl", [{"text": "aaaaaaaa"}])
    two = _jsonl(tmp_path / "code.jsonl", [{"text": "bbbbbbbb"}])
    assert build_corpus([one, two], tok).domains == ["stories", "code"]  # several files: the stem is the domain


def test_repetitive_windows_score_easier_and_the_stream_reports_its_stage():
    from quantaweave_b200.data.pipeline import Segment, TokenCorpus

    tok = CharTokenizer.build(["abcdefgh"], 16)
    text = "aaaaaaaa" + "abcdefgh"
    ds = WindowDataset(TokenCorpus(torch.tensor(tok.encode(text), dtype=torch.int32), [Segment("default", 0, 16)]),
                       7)
    assert len(ds) == 2
    for method in ("rarity", "entropy"):
        scores = difficulty_scores(ds, method, tok.vocab_size)
        assert scores[0] <= scores[1], method
    stream = BatchStream(ds, 4, seed=3, scores=difficulty_scores(ds, "entropy", tok.vocab_size),
                         curriculum=CurriculumConfig("entropy", start_fraction=0.5, steps=10))
    state = stream.state(5)
    assert state["samples_consumed"] == 20 and state["domain_weights"] == {"default": 1.0}
    assert 1 <= state["curriculum_stage"] <= 4


def test_an_empty_stream_is_refused(tmp_path):
    data = _jsonl(tmp_path / "d.jsonl", [{"text": "ab"}])
    ds = WindowDataset(build_corpus([data], CharTokenizer.build(["ab"], 8)), 32)
    assert len(ds) == 0
    with pytest.raises(ValueError):
        BatchStream(ds, 2)
