"""Best-effort regex PII redaction applied to rows before tokenisation (reference ``src/pii_redact.py``).

Matches e-mail addresses, separated phone numbers, US SSN shapes, 16-digit card shapes and IPv4 addresses and
replaces each with ``<CATEGORY>``. It is not a PII-detection model: expect misses and occasional false positives.
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field

_PATTERNS: dict[str, re.Pattern] = {
    "EMAIL": re.compile(r"[A-Za-z0-9._%+-]+@[A-Za-z0-9.-]+\.[A-Za-z]{2,}"),
    "PHONE": re.compile(r"(?<!\d)(?:\+?\d{1,3}[-.\s]?)?\(?\d{3}\)?[-.\s]\d{3}[-.\s]\d{4}(?!\d)"),
    "SSN": re.compile(r"(?<!\d)\d{3}-\d{2}-\d{4}(?!\d)"),
    "CREDIT_CARD": re.compile(r"(?<!\d)(?:\d{4}[-\s]){3}\d{4}(?!\d)"),
    "IPV4": re.compile(r"(?<!\d)(?:(?:25[0-5]|2[0-4]\d|1?\d?\d)\.){3}(?:25[0-5]|2[0-4]\d|1?\d?\d)(?!\d)"),
}


@dataclass
class PIIRedactor:
    counts: dict = field(default_factory=lambda: {name: 0 for name in _PATTERNS})

    def redact(self, text: str) -> str:
        for name, pattern in _PATTERNS.items():
            text, hits = pattern.subn(f"<{name}>", text)
            self.counts[name] += hits
        return text

    def report(self) -> dict:
        return dict(self.counts)

    def total(self) -> int:
        return sum(self.counts.values())
