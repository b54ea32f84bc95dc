"""Distillation from a teacher with a different tokenizer (for example a Hugging Face causal LM).

Behavioural parity with the reference ``src/cross_tokenizer.py`` (``HFTeacher`` :30-66, ``align_positions`` :77-94,
``first_char_matrix`` :97-106, ``uld_loss`` :106-112, ``marginal_kl`` :114-119, ``CrossTokenizerLoss`` :122-168).
Teacher and student read the same text. A student position supervises only where its token ends at the same
character offset as a teacher token (both then predict "what comes after this text"). Losses:

* ``marginal`` (character-level students, exact): the teacher's next-token distribution is collapsed onto each
  candidate token's first character, giving the teacher's next-character distribution; KL(teacher || student).
* ``uld`` (any student): L1 between the descending-sorted distributions (universal logit distillation), which needs
  no vocabulary mapping.

Documents split at ``<eos>``; each segment is scored on its own. B200 choice: all segments of a batch are scored by
the teacher in ONE padded forward (right padding, attention mask) instead of one forward per segment.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.nn.functional as F
from torch import Tensor

REPLACEMENT = "�"


class HFTeacher:
    """A Hugging Face causal LM (directory or hub id) scored on raw text; needs a fast tokenizer (char offsets)."""

    def __init__(self, path: str, device: torch.device, precision_dtype: Optional[torch.dtype] = None) -> None:
        try:
            from transformers import AutoModelForCausalLM, AutoTokenizer
        except ImportError as error:  # pragma: no cover - transformers is installed in this image
            raise RuntimeError("--hf-teacher needs the `transformers` package") from error
        self.tokenizer = AutoTokenizer.from_pretrained(path, use_fast=True)
        if not getattr(self.tokenizer, "is_fast", False):
            raise ValueError("the teacher needs a fast tokenizer: character offsets align it with the student")
        self.model = AutoModelForCausalLM.from_pretrained(path, torch_dtype=precision_dtype).to(device).eval()
        for p in self.model.parameters():
            p.requires_grad_(False)
        self.device = device
        self.vocab_size = self.model.get_output_embeddings().weight.size(0)
        cfg = self.model.config
        limit = getattr(cfg, "max_position_embeddings", None) or getattr(cfg, "n_positions", None)
        self.max_tokens = int(limit) if limit else 2048
        self._strings: Optional[list[str]] = None

    def token_strings(self) -> list[str]:
        if self._strings is None:
            self._strings = [self.tokenizer.decode([i]) for i in range(self.vocab_size)]
        return self._strings

    @torch.no_grad()
    def next_token_probs(self, text: str) -> tuple[Tensor, list[int]]:
        """(probs [T, V], end offset of each token); probs[k] predicts the token after token k."""
        probs, ends = self.next_token_probs_batch([text])
        return probs[0], ends[0]

    @torch.no_grad()
    def next_token_probs_batch(self, texts: Sequence[str]) -> tuple[list[Tensor], list[list[int]]]:
        enc = [self.tokenizer(t, add_special_tokens=False, return_offsets_mapping=True) for t in texts]
        ids = [e["input_ids"][: self.max_tokens] for e in enc]
        ends = [[int(b) for _, b in e["offset_mapping"][: self.max_tokens]] for e in enc]
        width = max((len(x) for x in ids), default=0)
        if width == 0:
            return [torch.zeros(0, self.vocab_size, device=self.device) for _ in texts], ends
        pad = self.tokenizer.pad_token_id if self.tokenizer.pad_token_id is not None else 0
        batch = torch.full((len(ids), width), pad, dtype=torch.long)
        mask = torch.zeros(len(ids), width, dtype=torch.long)
        for i, row in enumerate(ids):
            batch[i, : len(row)] = torch.tensor(row, dtype=torch.long)
            mask[i, : len(row)] = 1
        logits = self.model(input_ids=batch.to(self.device), attention_mask=mask.to(self.device)).logits.float()
        probs = logits.softmax(dim=-1)
        return [probs[i, : len(row)] for i, row in enumerate(ids)], ends


def student_pieces(tokenizer) -> list[str]:
    """The text each student token id stands for (``<eos>`` is empty, ``<unk>`` the replacement character)."""
    if tokenizer.kind == "char":
        pieces = [tokenizer.inverse.get(i, REPLACEMENT) for i in range(tokenizer.vocab_size)]
        pieces[tokenizer.unk_id] = REPLACEMENT
    else:
        pieces = [tokenizer.decode([i]) for i in range(tokenizer.vocab_size)]
    pieces[tokenizer.eos_id] = ""
    return pieces


def align_positions(piece_lengths: Sequence[int], teacher_ends: Sequence[int]) -> list[tuple[int, int]]:
    """(student position j, teacher position k) pairs that predict the same next event.

    Student position j (after token j) aligns with teacher token k when both end at the same character offset; when
    several teacher tokens end there the last one wins. The last student token has no successor."""
    last_at = {end: k for k, end in enumerate(teacher_ends)}
    pairs = []
    offset = 0
    for j, length in enumerate(piece_lengths[:-1]):
        offset += length
        if length and offset in last_at:
            pairs.append((j, last_at[offset]))
    return pairs


def first_char_matrix(teacher_strings: Sequence[str], student_tokenizer, device: torch.device,
                      width: Optional[int] = None) -> Tensor:
    """0/1 matrix [teacher vocab, width]: teacher token t starts with student character c."""
    cols = torch.tensor([student_tokenizer.vocab.get(s[0], student_tokenizer.unk_id) if s else student_tokenizer.unk_id
                         for s in teacher_strings], dtype=torch.long)
    matrix = torch.zeros(len(teacher_strings), width or student_tokenizer.vocab_size)
    matrix[torch.arange(len(teacher_strings)), cols] = 1.0
    return matrix.to(device)


def uld_loss(student_probs: Tensor, teacher_probs: Tensor) -> Tensor:
    """Mean L1 distance between the descending-sorted distributions, the shorter one zero-padded."""
    width = max(student_probs.size(-1), teacher_probs.size(-1))
    s = F.pad(student_probs.sort(dim=-1, descending=True).values, (0, width - student_probs.size(-1)))
    t = F.pad(teacher_probs.sort(dim=-1, descending=True).values, (0, width - teacher_probs.size(-1)))
    return (s - t).abs().sum(dim=-1).mean()


def marginal_kl(student_logits: Tensor, teacher_probs: Tensor, matrix: Tensor) -> Tensor:
    """KL(teacher's next-character distribution || student), averaged over the aligned positions."""
    return F.kl_div(F.log_softmax(student_logits.float(), dim=-1), teacher_probs @ matrix, reduction="batchmean")


class CrossTokenizerLoss:
    def __init__(self, teacher, student_tokenizer, mode: str = "auto") -> None:
        if mode == "auto":
            mode = "marginal" if student_tokenizer.kind == "char" else "uld"
        if mode not in {"marginal", "uld"}:
            raise ValueError("cross-tokenizer loss must be auto, marginal or uld")
        if mode == "marginal" and student_tokenizer.kind != "char":
            raise ValueError("the marginal loss is exact only for character-level students; use uld for BPE students")
        self.teacher, self.tokenizer, self.mode = teacher, student_tokenizer, mode
        self.pieces = student_pieces(student_tokenizer)
        self.matrix: Optional[Tensor] = None

    def segments(self, ids: Sequence[int]):
        """(start position, token ids) of every ``<eos>``-separated segment with at least two tokens."""
        start, current = 0, []
        for pos, tok in enumerate(list(ids) + [self.tokenizer.eos_id]):
            if tok == self.tokenizer.eos_id:
                if len(current) > 1:
                    yield start, current
                start, current = pos + 1, []
            else:
                current.append(tok)

    def __call__(self, student_logits: Tensor, batch: Tensor) -> tuple[Tensor, dict]:
        """``student_logits [B, L, V]``, ``batch [B, L]`` ids -> (loss, stats)."""
        work = []  # (row, start, ids, text)
        for b in range(batch.size(0)):
            for start, ids in self.segments(batch[b].tolist()):
                text = "".join(self.pieces[i] for i in ids)
                if self.tokenizer.kind != "char" and self.tokenizer.decode(ids) != text:
                    raise ValueError("student tokens do not decode to text piece by piece (byte-level splits); "
                                     "cross-tokenizer distillation needs tokens that are valid text on their own")
                work.append((b, start, ids, text))
        considered = sum(len(ids) - 1 for _, _, ids, _ in work)
        rows, cols, targets = [], [], []
        if work:
            if hasattr(self.teacher, "next_token_probs_batch"):
                all_probs, all_ends = self.teacher.next_token_probs_batch([w[3] for w in work])
            else:
                scored = [self.teacher.next_token_probs(w[3]) for w in work]
                all_probs, all_ends = [s[0] for s in scored], [s[1] for s in scored]
            for (b, start, ids, _), probs, ends in zip(work, all_probs, all_ends):
                for j, k in align_positions([len(self.pieces[i]) for i in ids], ends):
                    rows.append(b)
                    cols.append(start + j)
                    targets.append(probs[k])
        stats = {"aligned_positions": len(rows), "considered_positions": considered,
                 "aligned_fraction": len(rows) / considered if considered else 0.0, "mode": self.mode}
        if not rows:
            return student_logits.sum() * 0.0, stats
        logits = student_logits[torch.tensor(rows), torch.tensor(cols)]
        teacher_probs = torch.stack(targets).to(student_logits.device)
        if self.mode == "marginal":
            if self.matrix is None:
                self.matrix = first_char_matrix(self.teacher.token_strings(), self.tokenizer, student_logits.device,
                                                student_logits.size(-1))
            return marginal_kl(logits, teacher_probs, self.matrix), stats
        return uld_loss(F.softmax(logits.float(), dim=-1), teacher_probs), stats
