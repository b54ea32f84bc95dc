"""Tokenizers, domain-tagged token corpora, window datasets, curriculum, domain mixtures and batch streams.

The data formats and public names follow the reference's ``src/data_pipeline.py``: JSONL rows with an optional
``domain`` field; character, byte-level BPE and SentencePiece tokenizers with ``<unk>`` = 0 and ``<eos>`` = 1 and
their saved files; packed corpora as ``tokens.bin`` + ``meta.json`` + ``tokenizer/``.

Here a corpus is one flat token array cut into per-domain segments; windows of ``sequence_length + 1`` tokens are
laid out inside segments only; ``BatchStream.batch(step)`` is a pure function of (seed, step, rank layout), so a
resumed run draws exactly the windows an uninterrupted one would. ``SyntheticTokenStream`` (seeded uniform or Zipf
token ids, the benchmark inputs) follows the same ``batch(step)`` / ``state(step)`` contract.
"""

from __future__ import annotations

import copy
import hashlib
import itertools
import json
import math
import re
import unicodedata
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
    """All token ids in one flat array (a tensor, or a read-only memmap for packed corpora), cut into one segment per
    domain. Every document ends with ``<eos>``; segments never overlap."""

    def __init__(self, data, segments: list[Segment]) -> None:
        self._data = data
        self.segments = segments
        self.domains = list(dict.fromkeys(seg.domain for seg in segments))

    def read(self, start: int, stop: int) -> Tensor:
        piece = self._data[start:stop]
        if isinstance(piece, Tensor):
            return piece.long()
        import numpy as np

        return torch.from_numpy(np.array(piece, dtype=np.int64))

    def __len__(self) -> int:
        return sum(seg.length for seg in self.segments)


def _documents(paths: Sequence[Path], tokenizer, limit: Optional[int], redactor) -> Iterator[tuple[str, list[int]]]:
    """(domain, token ids ending with ``<eos>``) for every row."""
    for domain, text in read_rows(paths, limit, redactor):
        yield domain, tokenizer.encode(text) + [tokenizer.eos_id]


def build_corpus(paths: Sequence[Path], tokenizer, limit: Optional[int] = None, redactor=None) -> TokenCorpus:
    """Tokenise the rows in memory: the documents of each domain back to back, domains in order of first row."""
    per_domain: dict[str, list[int]] = {}
    for domain, ids in _documents(paths, tokenizer, limit, redactor):
        per_domain.setdefault(domain, []).extend(ids)
    lengths = [len(ids) for ids in per_domain.values()]
    offsets = [0, *itertools.accumulate(lengths)]
    segments = [Segment(domain, offsets[i], lengths[i]) for i, domain in enumerate(per_domain)]
    flat = [token for ids in per_domain.values() for token in ids]
    return TokenCorpus(torch.tensor(flat, dtype=torch.int32), segments)


class _Spool:
    """Token ids of one domain appended to a temporary file as they are produced (bounded memory)."""

    def __init__(self, path: Path, dtype) -> None:
        self.path, self.dtype, self.length = path, dtype, 0
        self.handle = path.open("wb")

    def add(self, ids: list[int]) -> None:
        import numpy as np

        np.asarray(ids, dtype=self.dtype).tofile(self.handle)
        self.length += len(ids)


def write_token_bin(paths: Sequence[Path], tokenizer, out_dir: Path, limit: Optional[int] = None,
                    redactor=None) -> dict:
    """Pack the rows into ``tokens.bin`` (uint16, or uint32 for vocabularies over 65,536 ids) with ``meta.json``
    describing the per-domain segments, and the tokenizer beside them, for memory-mapped training."""
    import numpy as np

    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    dtype = np.dtype(np.uint16 if tokenizer.vocab_size <= 1 << 16 else np.uint32)
    spools: dict[str, _Spool] = {}
    try:
        for domain, ids in _documents(paths, tokenizer, limit, redactor):
            if domain not in spools:
                spools[domain] = _Spool(out_dir / f".spool-{len(spools)}.bin", dtype)
            spools[domain].add(ids)
    finally:
        for spool in spools.values():
            spool.handle.close()
    segments, position = [], 0
    with (out_dir / "tokens.bin").open("wb") as packed:
        for domain, spool in spools.items():
            segments.append({"domain": domain, "start": position, "length": spool.length})
            position += spool.length
            packed.write(spool.path.read_bytes())
            spool.path.unlink()
    tokenizer.save(out_dir / "tokenizer")
    meta = {"format": 1, "dtype": dtype.name, "tokenizer": tokenizer.kind, "vocab_size": tokenizer.vocab_size,
            "eos_id": tokenizer.eos_id, "segments": segments, "total_tokens": position}
    (out_dir / "meta.json").write_text(json.dumps(meta, indent=2) + "\n")
    return meta


def load_token_bin(directory: Path) -> tuple[TokenCorpus, object]:
    """(corpus, tokenizer) of a packed directory; the tokens stay on disk, memory-mapped."""
    import numpy as np

    directory = Path(directory)
    meta = json.loads((directory / "meta.json").read_text())
    tokenizer = load_tokenizer(directory / "tokenizer")
    segments = [Segment(s["domain"], s["start"], s["length"]) for s in meta["segments"]]
    if not meta["total_tokens"]:
        return TokenCorpus(torch.empty(0, dtype=torch.int32), []), tokenizer
    return TokenCorpus(np.memmap(directory / "tokens.bin", dtype=np.dtype(meta["dtype"]), mode="r"), segments), tokenizer


# ------------------------------------------------------------------------------------------ windows
class WindowDataset(Dataset):
    """Consecutive, non-overlapping windows of ``sequence_length + 1`` tokens inside each domain's segment (a
    partial window at the end of a segment is dropped), so no window mixes two domains."""

    def __init__(self, corpus: TokenCorpus, sequence_length: int) -> None:
        self.corpus, self.window, self.domains = corpus, sequence_length + 1, corpus.domains
        counts = torch.tensor([seg.length // self.window for seg in corpus.segments], dtype=torch.long)
        firsts = torch.tensor([seg.start for seg in corpus.segments], dtype=torch.long)
        owners = torch.tensor([self.domains.index(seg.domain) for seg in corpus.segments], dtype=torch.long)
        total = int(counts.sum())
        segment_of = torch.repeat_interleave(torch.arange(len(corpus.segments)), counts)
        before = torch.cumsum(counts, 0) - counts  # windows in earlier segments
        rank_in_segment = torch.arange(total) - before[segment_of] if total else torch.zeros(0, dtype=torch.long)
        self.starts = firsts[segment_of] + rank_in_segment * self.window if total else torch.zeros(0, dtype=torch.long)
        self.window_domains = owners[segment_of] if total else torch.zeros(0, dtype=torch.long)

    def __len__(self) -> int:
        return int(self.starts.numel())

    def __getitem__(self, index: int) -> Tensor:
        if not 0 <= index < len(self):
            raise IndexError(index)
        first = int(self.starts[index])
        return self.corpus.read(first, first + self.window)

    def batch(self, indices: Sequence[int]) -> Tensor:
        return torch.stack([self[int(i)] for i in indices])

    def fingerprint(self) -> str:
        return hashlib.sha256(f"{len(self)}|{self.window}|{self.domains}".encode()).hexdigest()[:16]

    def _subset(self, keep: Tensor) -> "WindowDataset":
        part = copy.copy(self)
        part.starts, part.window_domains = self.starts[keep], self.window_domains[keep]
        return part

    def split_train_val(self, val_fraction: float = 0.02, seed: int = 0, min_val_windows_per_domain: int = 1):
        """(train, val) views that never share a window. Each domain gives ``val_fraction`` of its windows (at least
        ``min_val_windows_per_domain``) to validation, drawn by a generator seeded with ``seed``."""
        if not 0 < val_fraction < 1:
            raise ValueError("val_fraction must be in (0, 1)")
        gen = torch.Generator().manual_seed(seed)
        held = torch.zeros(len(self), dtype=torch.bool)
        for d, name in enumerate(self.domains):
            members = torch.nonzero(self.window_domains == d).flatten()
            if not members.numel():
                continue
            take = max(min_val_windows_per_domain, round(members.numel() * val_fraction))
            if take >= members.numel():
                raise ValueError(f"domain '{name}' has only {members.numel()} window(s), too few to both train on "
                                 f"and hold out {take} for validation; lower val_fraction or add data")
            held[members[torch.randperm(members.numel(), generator=gen)[:take]]] = True
        return self._subset(~held), self._subset(held)


class CharacterDataset(WindowDataset):
    def __init__(self, path: Path, vocab: dict[str, int], sequence_length: int, limit: Optional[int]) -> None:
        super().__init__(build_corpus([Path(path)], CharTokenizer(vocab), limit), sequence_length)


# ------------------------------------------------------------------------------------------ curriculum
def _blocks(dataset: WindowDataset, size: int) -> Iterator[tuple[int, Tensor]]:
    for first in range(0, len(dataset), size):
        yield first, dataset.batch(range(first, min(len(dataset), first + size)))


def difficulty_scores(dataset: WindowDataset, method: str, vocab_size: int, chunk: int = 4096) -> Tensor:
    """One difficulty per window, higher is harder: ``rarity`` is the mean surprisal of its tokens under the corpus
    unigram distribution, ``entropy`` the entropy of its own token histogram, ``uncommon`` the share of its tokens
    that are among the rarest tenth of the token types seen."""
    if method not in ("rarity", "entropy", "uncommon"):
        raise ValueError("curriculum method must be rarity, entropy or uncommon")
    frequency = torch.zeros(vocab_size, dtype=torch.float64)
    for _, rows in _blocks(dataset, chunk):
        frequency.index_add_(0, rows.flatten(), torch.ones(rows.numel(), dtype=torch.float64))
    surprisal = -torch.log((frequency / frequency.sum().clamp(min=1)).clamp(min=1e-12))
    present = frequency[frequency > 0]
    rare_limit = torch.quantile(present, 0.1) if present.numel() else torch.tensor(0.0, dtype=torch.float64)
    out = torch.empty(len(dataset), dtype=torch.float64)
    for first, rows in _blocks(dataset, chunk):
        span = slice(first, first + rows.size(0))
        if method == "rarity":
            out[span] = surprisal[rows].mean(dim=1)
        elif method == "uncommon":
            out[span] = (frequency[rows] <= rare_limit).double().mean(dim=1)
        else:
            for offset, row in enumerate(rows):
                _, counts = torch.unique(row, return_counts=True)
                p = counts.double() / row.numel()
                out[first + offset] = -(p * p.log()).sum()
    return out.float()


@dataclass
class CurriculumConfig:
    """Start from the easiest ``start_fraction`` of each domain's windows and widen linearly to all of them over
    ``steps`` steps (``steps`` 0: no curriculum)."""

    method: str = "rarity"
    start_fraction: float = 0.25
    steps: int = 0

    @property
    def enabled(self) -> bool:
        return self.steps > 0

    def fraction(self, step: int) -> float:
        if not self.enabled:
            return 1.0
        progress = min(1.0, step / self.steps)
        return self.start_fraction + (1.0 - self.start_fraction) * progress

    def stage(self, step: int, tiers: int = 4) -> int:
        """Which quarter (by default) of the difficulty range the sampler has reached, 1..tiers."""
        return max(1, math.ceil(self.fraction(step) * tiers - 1e-9))


_WEIGHT_ITEM = re.compile(r"\s*([^=,\s][^=,]*?)\s*=\s*([^,]+?)\s*$")


def parse_domain_weights(spec: Optional[str]) -> Optional[dict[str, float]]:
    """``"prose=3, code=1"`` -> ``{"prose": 3.0, "code": 1.0}``; None for an empty spec."""
    if not spec:
        return None
    weights = {}
    for item in spec.split(","):
        match = _WEIGHT_ITEM.match(item)
        if match is None:
            raise ValueError(f"bad domain weight '{item}', expected name=weight")
        weights[match[1]] = float(match[2])
    if any(w < 0 for w in weights.values()):
        raise ValueError("domain weights must be non-negative")
    return weights


class DomainMixture:
    """Sampling weights per domain, fixed or blended linearly from ``start`` to ``end`` over ``steps`` steps."""

    def __init__(self, domains: Sequence[str], start: dict[str, float], end: Optional[dict[str, float]] = None,
                 steps: int = 0):
        self.domains = list(domains)
        self.start = self._vector(start)
        self.end = self._vector(end) if end else None
        self.steps = steps

    def _vector(self, weights: dict[str, float]) -> Tensor:
        unknown = sorted(set(weights) - set(self.domains))
        if unknown:
            raise ValueError(f"unknown domains {unknown}; dataset has {self.domains}")
        missing = sorted(set(self.domains) - set(weights))
        if missing:
            raise ValueError(f"domain weights must cover every domain; missing {missing}")
        vector = torch.tensor([weights[d] for d in self.domains], dtype=torch.double)
        if vector.sum() <= 0:
            raise ValueError("domain weights must not all be zero")
        return vector / vector.sum()

    def weights(self, step: int) -> Tensor:
        if self.end is None or self.steps <= 0:
            return self.start.clone()
        t = min(1.0, step / self.steps)
        blend = torch.lerp(self.start, self.end, t)
        return blend / blend.sum()


# ------------------------------------------------------------------------------------------ batch streams
def _step_seed(seed: int, step: int) -> int:
    """A generator seed for (run seed, step): the same pair always gives the same batch, on every rank."""
    return (seed * 0x9E3779B1 + step * 0x85EBCA77 + 1) % (1 << 62)


class BatchStream:
    """``batch(step)`` draws one global batch from a generator seeded by (seed, step) alone and gives each rank its
    own slice, so a resumed or differently launched run sees exactly the same windows at every step.

    Each sample first picks a domain (by the mixture, else in proportion to the domain's windows), then one of the
    domain's windows; with a curriculum only the easiest ``fraction(step)`` of that domain's windows can be picked."""

    def __init__(self, dataset: WindowDataset, batch_size: int, seed: int = 0, scores: Optional[Tensor] = None,
                 curriculum: Optional[CurriculumConfig] = None, mixture: Optional[DomainMixture] = None,
                 rank: int = 0, world_size: int = 1) -> None:
        if len(dataset) == 0:
            raise ValueError("dataset holds fewer tokens than one training window")
        if curriculum is not None and curriculum.enabled and scores is None:
            raise ValueError("a curriculum needs difficulty scores")
        self.dataset, self.batch_size, self.seed = dataset, batch_size, seed
        self.curriculum = curriculum or CurriculumConfig()
        self.mixture = mixture
        self.rank, self.world_size = rank, world_size
        self.pools = []  # per domain: its windows, easiest first when there are scores
        for d in range(len(dataset.domains)):
            members = torch.nonzero(dataset.window_domains == d).flatten()
            if scores is not None and members.numel():
                members = members[torch.argsort(scores[members], stable=True)]
            self.pools.append(members)
        self.natural = torch.tensor([p.numel() for p in self.pools], dtype=torch.double)
        self._flat = torch.cat(self.pools)
        self._pool_start = torch.cumsum(self.natural.long(), 0) - self.natural.long()

    @property
    def num_domains(self) -> int:
        return len(self.dataset.domains)

    def domain_weights(self, step: int) -> Tensor:
        base = self.mixture.weights(step) if self.mixture is not None else self.natural
        weights = torch.where(self.natural > 0, base, torch.zeros_like(base))
        if weights.sum() <= 0:
            raise ValueError("no sampleable domain has non-zero weight")
        return weights / weights.sum()

    def batch(self, step: int) -> tuple[Tensor, Tensor]:
        count = self.batch_size * self.world_size
        gen = torch.Generator().manual_seed(_step_seed(self.seed, step))
        domains = torch.multinomial(self.domain_weights(step), count, replacement=True, generator=gen)
        reach = torch.ceil(self.curriculum.fraction(step) * self.natural[domains]).long().clamp(min=1)
        position = (torch.rand(count, generator=gen, dtype=torch.double) * reach).long().clamp(max=reach - 1)
        windows = self._flat[self._pool_start[domains] + position]
        mine = slice(self.rank * self.batch_size, (self.rank + 1) * self.batch_size)
        return self.dataset.batch(windows[mine].tolist()), domains[mine]

    def state(self, step: int) -> dict:
        curriculum = self.curriculum
        return {"seed": self.seed, "step": step, "samples_consumed": step * self.batch_size * self.world_size,
                "fingerprint": self.dataset.fingerprint(), "curriculum_fraction": curriculum.fraction(step),
                "curriculum_stage": curriculum.stage(step) if curriculum.enabled else None,
                "domain_weights": dict(zip(self.dataset.domains, map(float, self.domain_weights(step))))}


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
        gen = torch.Generator().manual_seed(_step_seed(self.seed, step))
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
