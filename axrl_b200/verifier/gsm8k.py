"""GSM8K answer extraction and scoring (strict '#### <number>' or last number; reference ``axrl/verifier/gsm8k.py:13-80``)."""

from __future__ import annotations

import re

from axrl_b200.verifier.base_verifier import BaseVerifier

_STRICT = re.compile(r"#### (\-?[0-9\.\,]+)")
_NUM = re.compile(r"(\-?[0-9\.\,]+)")


def extract_solution(text: str, method: str = "strict") -> str | None:
    if method == "strict":
        m = _STRICT.findall(text)
        return m[-1].replace(",", "").replace("$", "") if m else None
    nums = [n for n in _NUM.findall(text) if n not in ("", ".")]
    return nums[-1].replace(",", "").rstrip(".") if nums else None


def compute_score(text: str, ground_truth: str, method: str = "strict", format_score: float = 0.0, score: float = 1.0) -> float:
    ans = extract_solution(text, method)
    if ans is None:
        return 0.0
    try:
        return score if abs(float(ans) - float(str(ground_truth).replace(",", ""))) < 1e-6 else format_score
    except ValueError:
        return score if ans == ground_truth else format_score


class GSM8KVerifier(BaseVerifier):
    def __init__(self, method: str = "flexible") -> None:
        self.method = method

    def verify(self, response: str, answer: str) -> float:
        return compute_score(response, answer, self.method)
