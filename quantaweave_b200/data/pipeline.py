"""Tokenizers, domain-tagged token corpora, window datasets, curriculum, domain mixtures and batch streams.

Behavioural parity with the reference ``src/data_pipeline.py``:

* JSONL rows with an optional ``domain`` field (``read_rows`` :32); char / byte-level BPE / SentencePiece tokenizers
  with ``<unk>``=0, ``<eos>``=1 (:55-198); per-domain token corpora in memory or memmapped from ``tokens.bin`` +
  ``meta.json`` (:234-335); non-overlapping ``seq+1`` windows that never cross a domain (:338-409);
  curriculum difficulty scores (:420); domain mixtures (:490).
* ``BatchStream.batch(step)`` is a pure function of (seed, step, rank layout): a ``torch.Generator`` seeded with
  ``seed * 1_000_003 + step`` draws one global batch and each rank takes its disjoint slice (:517-590). The same
  seeding rule is kept so that resumed runs draw the same windows.

Additions: ``SyntheticTokenStream`` (seeded uniform or Zipf token ids, the benchmark inputs) with the same
``batch(step)`` / ``state(step)`` contract, and a pinned-host staging helper for the end-to-end bench path.
"""

from __future__ import annotations

import hashlib
import json
import math
import shutil
import unicodedata
from array import array
from dataclasses import dataclass
from pathlib import Path
from typing import Iterable, Iterator, Optional, Sequence

import torch
from torch import Tensor
from torch.utils.data import Dataset

SPECIAL_TOKENS = ("<unk>", "<eos>")


# ------------------------------------------------------------------------------------------ rows
def extract_text(row: dict) -> str:
    for key in ("teacher_text", "completion", "text"):
        value = row.get(key)
        if value:
            return value
    return row.get("prompt", "") + row.get("response", "")


def read_rows(paths: Sequence[Path], limit: Optional[int] = None, redactor=None) -> Iterator[tuple[str, str]]:
    """Yield ``(domain, text)``; ``limit`` caps rows per file; the domain defaults to ``default`` (one file) or
    the file stem (several files)."""
    paths = list(paths)
    for path in paths:
        fallback = "default" if len(paths) == 1 else Path(path).stem
        with Path(path).open(encoding="utf-8") as handle:
            for number, line in enumerate(handle):
                if limit is not None and number >= limit:
                    break
                if not line.strip():
                    continue
                row = json.loads(line)
                text = extract_text(row)
                if not text:
                    continue
                if redactor is not None:
                    text = redactor.redact(text)
                yield str(row.get("domain") or fallback), text


# ------------------------------------------------------------------------------------------ tokenizers
class CharTokenizer:
    kind = "char"

    def __init__(self, vocab: dict[str, int]) -> None:
        self.vocab = dict(vocab)
        self.unk_id = self.vocab["<unk>"]
        self.eos_id = self.vocab["<eos>"]
        self.inverse = {index: token for token, index in self.vocab.items()}

    @property
    def vocab_size(self) -> int:
        return max(self.vocab.values()) + 1

    @classmethod
    def build(cls, texts: Iterable[str], vocab_size: int) -> "CharTokenizer":
        counts: dict[str, int] = {}
        for text in texts:
            for ch in text:
                counts[ch] = counts.get(ch, 0) + 1
        reserved = {tok: i for i, tok in enumerate(SPECIAL_TOKENS)}
        ranked = sorted(counts, key=counts.get, reverse=True)[: max(0, vocab_size - len(reserved))]
        vocab = dict(reserved)
        for offset, ch in enumerate(ranked):
            vocab[ch] = offset + len(reserved)
        return cls(vocab)

    def encode(self, text: str) -> list[int]:
        get, unk = self.vocab.get, self.unk_id
        return [get(ch, unk) for ch in text]

    def decode(self, ids: Iterable[int]) -> str:
        return "".join(self.inverse.get(int(i), "?") for i in ids)

    def save(self, directory: Path) -> None:
        directory = Path(directory)
        directory.mkdir(parents=True, exist_ok=True)
        (directory / "vocab.json").write_text(json.dumps(self.vocab, ensure_ascii=False, indent=2) + "\n")
        (directory / "tokenizer_meta.json").write_text(json.dumps({"type": "char"}) + "\n")


class BPETokenizer:
    """Byte-level BPE trained with the ``tokenizers`` library."""

    kind = "bpe"

    def __init__(self, tokenizer) -> None:
        self.tokenizer = tokenizer
        self.unk_id = tokenizer.token_to_id("<unk>")
        self.eos_id = tokenizer.token_to_id("<eos>")

    @property
    def vocab_size(self) -> int:
        return self.tokenizer.get_vocab_size()

    @classmethod
    def train(cls, texts: Iterable[str], vocab_size: int) -> "BPETokenizer":
        from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers

        floor = 256 + len(SPECIAL_TOKENS)
        if vocab_size < floor:
            raise ValueError(f"byte-level BPE needs a vocab size of at least {floor}, got {vocab_size}")
        tok = Tokenizer(models.BPE(unk_token="<unk>"))
        tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
        tok.decoder = decoders.ByteLevel()
        trainer = trainers.BpeTrainer(vocab_size=vocab_size, special_tokens=list(SPECIAL_TOKENS),
                                      initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
        tok.train_from_iterator(texts, trainer=trainer)
        return cls(tok)

    def encode(self, text: str) -> list[int]:
        return self.tokenizer.encode(text).ids

    def decode(self, ids: Iterable[int]) -> str:
        return self.tokenizer.decode([int(i) for i in ids])

    def save(self, directory: Path) -> None:
        directory = Path(directory)
        directory.mkdir(parents=True, exist_ok=True)
        self.tokenizer.save(str(directory / "tokenizer.json"))
        (directory / "tokenizer_meta.json").write_text(json.dumps({"type": "bpe"}) + "\n")

    @classmethod
    def load(cls, directory: Path) -> "BPETokenizer":
        from tokenizers import Tokenizer

        return cls(Tokenizer.from_file(str(Path(directory) / "tokenizer.json")))


class SentencePieceTokenizer:
    """SentencePiece (unigram or BPE) with ``<unk>``=0 and ``<eos>``=1."""

    kind = "sentencepiece"

    def __init__(self, processor) -> None:
        self.processor = processor
        self.unk_id = processor.unk_id()
        self.eos_id = processor.piece_to_id("<eos>")

    @property
    def vocab_size(self) -> int:
        return self.processor.get_piece_size()

    @classmethod
    def train(cls, texts: Iterable[str], vocab_size: int, algorithm: str = "unigram") -> "SentencePieceTokenizer":
        import io

        import sentencepiece as spm

        if algorithm not in {"unigram", "bpe"}:
            raise ValueError("algorithm must be unigram or bpe")
        model = io.BytesIO()
        spm.SentencePieceTrainer.train(
            sentence_iterator=iter(list(texts)), model_writer=model, vocab_size=vocab_size, model_type=algorithm,
            unk_id=0, bos_id=-1, eos_id=1, pad_id=-1, eos_piece="<eos>", unk_piece="<unk>",
            character_coverage=1.0, hard_vocab_limit=False, minloglevel=2,
        )
        processor = spm.SentencePieceProcessor(model_proto=model.getvalue())
        return cls(processor)

    def encode(self, text: str) -> list[int]:
        return list(self.processor.encode(text))

    def decode(self, ids: Iterable[int]) -> str:
        return self.processor.decode([int(i) for i in ids])

    def save(self, directory: Path) -> None:
        directory = Path(directory)
        directory.mkdir(parents=True, exist_ok=True)
        (directory / "tokenizer.model").write_bytes(self.processor.serialized_model_proto())
        (directory / "tokenizer_meta.json").write_text(json.dumps({"type": "sentencepiece"}) + "\n")

    @classmethod
    def load(cls, directory: Path) -> "SentencePieceTokenizer":
        import sentencepiece as spm

        return cls(spm.SentencePieceProcessor(model_file=str(Path(directory) / "tokenizer.model")))


def load_tokenizer(directory: Path):
    directory = Path(directory)
    meta_path = directory / "tokenizer_meta.json"
    kind = json.loads(meta_path.read_text())["type"] if meta_path.exists() else None
    if kind == "bpe" or (kind is None and (directory / "tokenizer.json").exists()):
        return BPETokenizer.load(directory)
    if kind == "sentencepiece" or (kind is None and (directory / "tokenizer.model").exists()):
        return SentencePieceTokenizer.load(directory)
    return CharTokenizer(json.loads((directory / "vocab.json").read_text()))


TOKEN_CLASS_NAMES = ("special", "letter", "digit", "space", "punct", "other")


def token_classes(tokenizer) -> tuple[Tensor, list[str]]:
    """Coarse class of every token id for routing-specialisation maps, as ``(class index per id [vocab], names)``
    with the names special, letter, digit, space, punct and other (reference ``src/data_pipeline.py:199-223``).
    A token is judged by the first visible character of its text; all-whitespace tokens are ``space``."""
    names = list(TOKEN_CLASS_NAMES)
    classes = torch.full((tokenizer.vocab_size,), names.index("other"), dtype=torch.long)
    for index in range(tokenizer.vocab_size):
        if index in (tokenizer.unk_id, tokenizer.eos_id):
            classes[index] = names.index("special")
            continue
        text = tokenizer.decode([index])
        stripped = text.strip()
        if not stripped:
            label = "space" if text else "other"
        elif stripped[0].isalpha():
            label = "letter"
        elif stripped[0].isdigit():
            label = "digit"
        elif unicodedata.category(stripped[0])[0] in "PS":
            label = "punct"
        else:
            label = "other"
        classes[index] = names.index(label)
    return classes, names


# ------------------------------------------------------------------------------------------ corpora
@dataclass
class Segment:
    domain: str
    start: int
    length: int


class TokenCorpus:
    """One flat token stream split into per-domain segments (in memory or memmapped)."""

    def __init__(self, data, segments: list[Segment]) -> None:
        self._data = data
        self.segments = segments
        self.domains: list[str] = []
        for seg in segments:
            if seg.domain not in self.domains:
                self.domains.append(seg.domain)

    def read(self, start: int, stop: int) -> Tensor:
        if isinstance(self._data, Tensor):
            return self._data[start:stop].long()
        import numpy as np

        return torch.from_numpy(np.asarray(self._data[start:stop], dtype=np.int64))

    def __len__(self) -> int:
        return sum(seg.length for seg in self.segments)


def build_corpus(paths: Sequence[Path], tokenizer, limit: Optional[int] = None, redactor=None) -> TokenCorpus:
    """Tokenise JSONL rows into per-domain streams, each document followed by ``<eos>``."""
    streams: dict[str, array] = {}
    for domain, text in read_rows(paths, limit, redactor):
        stream = streams.setdefault(domain, array("i"))
        stream.extend(tokenizer.encode(text))
        stream.append(tokenizer.eos_id)
    joined = array("i")
    segments = []
    for domain, stream in streams.items():
        segments.append(Segment(domain, len(joined), len(stream)))
        joined.extend(stream)
    data = torch.tensor(joined, dtype=torch.int32) if len(joined) else torch.empty(0, dtype=torch.int32)
    return TokenCorpus(data, segments)


def write_token_bin(paths: Sequence[Path], tokenizer, out_dir: Path, limit: Optional[int] = None, redactor=None) -> dict:
    """Tokenise JSONL into a memmappable ``tokens.bin`` (uint16/uint32) plus ``meta.json`` and the tokenizer."""
    import numpy as np

    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    dtype = np.uint16 if tokenizer.vocab_size <= 2 ** 16 else np.uint32
    parts: dict[str, Path] = {}
    handles: dict = {}
    lengths: dict[str, int] = {}
    try:
        for domain, text in read_rows(paths, limit, redactor):
            if domain not in handles:
                parts[domain] = out_dir / f".tokens.{len(parts)}.part"
                handles[domain] = parts[domain].open("wb")
                lengths[domain] = 0
            ids = np.asarray(tokenizer.encode(text) + [tokenizer.eos_id], dtype=dtype)
            ids.tofile(handles[domain])
            lengths[domain] += int(ids.size)
    finally:
        for handle in handles.values():
            handle.close()
    segments = []
    itemsize = np.dtype(dtype).itemsize
    with (out_dir / "tokens.bin").open("wb") as target:
        for domain, part in parts.items():
            segments.append({"domain": domain, "start": target.tell() // itemsize, "length": lengths[domain]})
            with part.open("rb") as source:
                shutil.copyfileobj(source, target)
            part.unlink()
    tokenizer.save(out_dir / "tokenizer")
    meta = {"format": 1, "dtype": np.dtype(dtype).name, "tokenizer": tokenizer.kind, "vocab_size": tokenizer.vocab_size,
            "eos_id": tokenizer.eos_id, "segments": segments, "total_tokens": sum(lengths.values())}
    (out_dir / "meta.json").write_text(json.dumps(meta, indent=2) + "\n")
    return meta


def load_token_bin(directory: Path) -> tuple[TokenCorpus, object]:
    import numpy as np

    directory = Path(directory)
    meta = json.loads((directory / "meta.json").read_text())
    tokenizer = load_tokenizer(directory / "tokenizer")
    if meta["total_tokens"] == 0:
        return TokenCorpus(torch.empty(0, dtype=torch.int32), []), tokenizer
    data = np.memmap(directory / "tokens.bin", dtype=np.dtype(meta["dtype"]), mode="r")
    segments = [Segment(s["domain"], s["start"], s["length"]) for s in meta["segments"]]
    return TokenCorpus(data, segments), tokenizer


# ------------------------------------------------------------------------------------------ windows
class WindowDataset(Dataset):
    """Non-overlapping windows of ``sequence_length + 1`` tokens that never cross a domain boundary."""

    def __init__(self, corpus: TokenCorpus, sequence_length: int) -> None:
        self.corpus = corpus
        self.window = sequence_length + 1
        self.domains = corpus.domains
        starts, owners = [], []
        for seg in corpus.segments:
            count = seg.length // self.window
            starts.append(seg.start + torch.arange(count, dtype=torch.long) * self.window)
            owners.append(torch.full((count,), self.domains.index(seg.domain), dtype=torch.long))
        self.starts = torch.cat(starts) if starts else torch.empty(0, dtype=torch.long)
        self.window_domains = torch.cat(owners) if owners else torch.empty(0, dtype=torch.long)

    def __len__(self) -> int:
        return int(self.starts.numel())

    def __getitem__(self, index: int) -> Tensor:
        if not 0 <= index < len(self):
            raise IndexError(index)
        start = int(self.starts[index])
        return self.corpus.read(start, start + self.window)

    def batch(self, indices: Sequence[int]) -> Tensor:
        return torch.stack([self[int(i)] for i in indices])

    def fingerprint(self) -> str:
        return hashlib.sha256(f"{len(self)}|{self.window}|{self.domains}".encode()).hexdigest()[:16]

    @classmethod
    def _view(cls, corpus, window, domains, starts, window_domains) -> "WindowDataset":
        view = cls.__new__(cls)
        view.corpus, view.window, view.domains = corpus, window, domains
        view.starts, view.window_domains = starts, window_domains
        return view

    def split_train_val(self, val_fraction: float = 0.02, seed: int = 0, min_val_windows_per_domain: int = 1):
        """Domain-stratified deterministic (train, val) split; the two views never overlap."""
        if not 0 < val_fraction < 1:
            raise ValueError("val_fraction must be in (0, 1)")
        gen = torch.Generator().manual_seed(seed)
        train_parts, val_parts = [], []
        for d in range(len(self.domains)):
            where = (self.window_domains == d).nonzero(as_tuple=True)[0]
            if where.numel() == 0:
                continue
            shuffled = where[torch.randperm(where.numel(), generator=gen)]
            held = max(min_val_windows_per_domain, round(where.numel() * val_fraction))
            if held >= where.numel():
                raise ValueError(f"domain '{self.domains[d]}' has only {where.numel()} window(s), too few to both "
                                 f"train on and hold out {held} for validation; lower val_fraction or add data")
            val_parts.append(shuffled[:held])
            train_parts.append(shuffled[held:])
        tr = torch.cat(train_parts).sort().values
        va = torch.cat(val_parts).sort().values
        return (self._view(self.corpus, self.window, self.domains, self.starts[tr], self.window_domains[tr]),
                self._view(self.corpus, self.window, self.domains, self.starts[va], self.window_domains[va]))


class CharacterDataset(WindowDataset):
    def __init__(self, path: Path, vocab: dict[str, int], sequence_length: int, limit: Optional[int]) -> None:
        super().__init__(build_corpus([Path(path)], CharTokenizer(vocab), limit), sequence_length)


# ------------------------------------------------------------------------------------------ curriculum
def difficulty_scores(dataset: WindowDataset, method: str, vocab_size: int, chunk: int = 4096) -> Tensor:
    """Per-window difficulty (higher = harder): ``rarity`` mean -log unigram frequency, ``entropy`` histogram
    entropy, ``uncommon`` share of tokens in the rarest 10% by corpus frequency."""
    if method not in {"rarity", "entropy", "uncommon"}:
        raise ValueError("curriculum method must be rarity, entropy or uncommon")
    total = len(dataset)
    counts = torch.zeros(vocab_size, dtype=torch.float64)
    for lo in range(0, total, chunk):
        rows = dataset.batch(range(lo, min(total, lo + chunk)))
        counts += torch.bincount(rows.reshape(-1), minlength=vocab_size).double()
    freq = counts / counts.sum().clamp(min=1)
    neg_log = -(freq.clamp_min(1e-12)).log()
    seen = counts[counts > 0]
    cutoff = torch.quantile(seen, 0.1) if seen.numel() else torch.tensor(0.0, dtype=torch.float64)
    scores = torch.empty(total, dtype=torch.float64)
    for lo in range(0, total, chunk):
        rows = dataset.batch(range(lo, min(total, lo + chunk)))
        if method == "rarity":
            scores[lo: lo + len(rows)] = neg_log[rows].mean(dim=1)
        elif method == "uncommon":
            scores[lo: lo + len(rows)] = (counts[rows] <= cutoff).double().mean(dim=1)
        else:
            for r, toks in enumerate(rows):
                hist = torch.bincount(toks).double()
                p = hist[hist > 0] / toks.numel()
                scores[lo + r] = -(p * p.log()).sum()
    return scores.float()


@dataclass
class CurriculumConfig:
    method: str = "rarity"
    start_fraction: float = 0.25
    steps: int = 0

    @property
    def enabled(self) -> bool:
        return self.steps > 0

    def fraction(self, step: int) -> float:
        if not self.enabled:
            return 1.0
        return min(1.0, self.start_fraction + (1.0 - self.start_fraction) * step / self.steps)

    def stage(self, step: int, tiers: int = 4) -> int:
        return max(1, math.ceil(self.fraction(step) * tiers - 1e-9))


def parse_domain_weights(spec: Optional[str]) -> Optional[dict[str, float]]:
    if not spec:
        return None
    weights: dict[str, float] = {}
    for item in spec.split(","):
        name, _, value = item.partition("=")
        name = name.strip()
        if not name or not value:
            raise ValueError(f"bad domain weight '{item}', expected name=weight")
        weights[name] = float(value)
        if weights[name] < 0:
            raise ValueError("domain weights must be non-negative")
    return weights


class DomainMixture:
    def __init__(self, domains: Sequence[str], start: dict[str, float], end: Optional[dict[str, float]] = None, steps: int = 0):
        for weights in (start, end or {}):
            unknown = set(weights) - set(domains)
            if unknown:
                raise ValueError(f"unknown domains {sorted(unknown)}; dataset has {list(domains)}")
            missing = set(domains) - set(weights)
            if weights and missing:
                raise ValueError(f"domain weights must cover every domain; missing {sorted(missing)}")
        self.domains = list(domains)
        self.start = torch.tensor([start[d] for d in domains], dtype=torch.double)
        self.end = torch.tensor([end[d] for d in domains], dtype=torch.double) if end else None
        self.steps = steps
        if self.start.sum() <= 0 or (self.end is not None and self.end.sum() <= 0):
            raise ValueError("domain weights must not all be zero")

    def weights(self, step: int) -> Tensor:
        if self.end is None or self.steps <= 0:
            return self.start / self.start.sum()
        mix = min(1.0, step / self.steps)
        blended = (1 - mix) * self.start / self.start.sum() + mix * self.end / self.end.sum()
        return blended / blended.sum()


# ------------------------------------------------------------------------------------------ batch streams
class BatchStream:
    """Deterministic batches: ``batch(step)`` depends only on (seed, step, rank, world_size)."""

    def __init__(self, dataset: WindowDataset, batch_size: int, seed: int = 0, scores: Optional[Tensor] = None,
                 curriculum: Optional[CurriculumConfig] = None, mixture: Optional[DomainMixture] = None,
                 rank: int = 0, world_size: int = 1) -> None:
        if len(dataset) == 0:
            raise ValueError("dataset holds fewer tokens than one training window")
        if curriculum is not None and curriculum.enabled and scores is None:
            raise ValueError("a curriculum needs difficulty scores")
        self.dataset = dataset
        self.batch_size = batch_size
        self.seed = seed
        self.curriculum = curriculum or CurriculumConfig()
        self.mixture = mixture
        self.rank, self.world_size = rank, world_size
        self.pools: list[Tensor] = []
        for d in range(len(dataset.domains)):
            idx = (dataset.window_domains == d).nonzero(as_tuple=True)[0]
            if scores is not None and idx.numel():
                idx = idx[torch.argsort(scores[idx], stable=True)]
            self.pools.append(idx)
        self.natural = torch.tensor([p.numel() for p in self.pools], dtype=torch.double)

    @property
    def num_domains(self) -> int:
        return len(self.dataset.domains)

    def domain_weights(self, step: int) -> Tensor:
        weights = (self.mixture.weights(step) if self.mixture is not None else self.natural).clone()
        weights[self.natural == 0] = 0
        if weights.sum() <= 0:
            raise ValueError("no sampleable domain has non-zero weight")
        return weights / weights.sum()

    def batch(self, step: int) -> tuple[Tensor, Tensor]:
        total = self.batch_size * self.world_size
        gen = torch.Generator().manual_seed(self.seed * 1_000_003 + step)
        domains = torch.multinomial(self.domain_weights(step), total, replacement=True, generator=gen)
        uniform = torch.rand(total, generator=gen, dtype=torch.double)
        fraction = self.curriculum.fraction(step)
        chosen = []
        for d, u in zip(domains.tolist(), uniform.tolist()):
            pool = self.pools[d]
            reach = max(1, math.ceil(fraction * pool.numel()))
            chosen.append(int(pool[min(int(u * reach), reach - 1)]))
        mine = slice(self.rank * self.batch_size, (self.rank + 1) * self.batch_size)
        return self.dataset.batch(chosen[mine]), domains[mine]

    def state(self, step: int) -> dict:
        return {
            "seed": self.seed,
            "step": step,
            "samples_consumed": step * self.batch_size * self.world_size,
            "fingerprint": self.dataset.fingerprint(),
            "curriculum_fraction": self.curriculum.fraction(step),
            "curriculum_stage": self.curriculum.stage(step) if self.curriculum.enabled else None,
            "domain_weights": {d: float(w) for d, w in zip(self.dataset.domains, self.domain_weights(step))},
        }


class SyntheticTokenStream:
    """Seeded synthetic token windows ``[batch, seq+1]`` (uniform or Zipf over the vocabulary).

    Same contract as ``BatchStream``: ``batch(step)`` is a pure function of (seed, step, rank layout); every rank
    takes a disjoint slice of one global draw, so runs resume and scale deterministically. Zipf ids are drawn by
    inverse-CDF sampling of ``p(r) ∝ r^-s`` over ranks ``1..vocab``; rank ``r`` maps to token ``r - 1``.
    """

    def __init__(self, vocab_size: int, sequence_length: int, batch_size: int, seed: int = 0,
                 distribution: str = "uniform", zipf_s: float = 1.1, rank: int = 0, world_size: int = 1) -> None:
        if distribution not in {"uniform", "zipf"}:
            raise ValueError("distribution must be uniform or zipf")
        self.vocab_size = vocab_size
        self.sequence_length = sequence_length
        self.batch_size = batch_size
        self.seed = seed
        self.distribution = distribution
        self.zipf_s = zipf_s
        self.rank, self.world_size = rank, world_size
        self.domains = ["synthetic"]
        if distribution == "zipf":
            ranks = torch.arange(1, vocab_size + 1, dtype=torch.float64)
            weights = ranks.pow(-zipf_s)
            self._cdf = torch.cumsum(weights / weights.sum(), dim=0)
            self._cdf[-1] = 1.0

    @property
    def num_domains(self) -> int:
        return 1

    def global_batch(self, step: int) -> Tensor:
        total = self.batch_size * self.world_size
        gen = torch.Generator().manual_seed(self.seed * 1_000_003 + step)
        shape = (total, self.sequence_length + 1)
        if self.distribution == "uniform":
            return torch.randint(0, self.vocab_size, shape, generator=gen, dtype=torch.long)
        u = torch.rand(shape, generator=gen, dtype=torch.float64)
        return torch.searchsorted(self._cdf, u).clamp_(max=self.vocab_size - 1)

    def batch(self, step: int) -> tuple[Tensor, Tensor]:
        tokens = self.global_batch(step)
        mine = tokens[self.rank * self.batch_size:(self.rank + 1) * self.batch_size]
        return mine.contiguous(), torch.zeros(self.batch_size, dtype=torch.long)

    def fingerprint(self) -> str:
        spec = f"{self.vocab_size}|{self.sequence_length}|{self.distribution}|{self.zipf_s}"
        return hashlib.sha256(spec.encode()).hexdigest()[:16]

    def state(self, step: int) -> dict:
        return {"seed": self.seed, "step": step, "samples_consumed": step * self.batch_size * self.world_size,
                "fingerprint": self.fingerprint(), "distribution": self.distribution, "zipf_s": self.zipf_s,
                "curriculum_fraction": 1.0, "curriculum_stage": None, "domain_weights": {"synthetic": 1.0}}
