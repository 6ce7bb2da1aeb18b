"""Boxed-answer math scoring with light normalisation (reference ``axrl/verifier/math_reward.py:13-229``)."""

from __future__ import annotations

import re

from axrl_b200.verifier.base_verifier import BaseVerifier


def last_boxed(text: str) -> str | None:
    i = text.rfind("\\boxed")
    if i < 0:
        i = text.rfind("\\fbox")
        if i < 0:
            return None
    j = text.find("{", i)
    if j < 0:
        return None
    depth = 0
    for k in range(j, len(text)):
        if text[k] == "{":
            depth += 1
        elif text[k] == "}":
            depth -= 1
            if depth == 0:
                return text[j + 1:k]
    return None


def normalize(ans: str) -> str:
    s = ans.strip().replace(" ", "").replace("\\!", "").replace("$", "")
    s = re.sub(r"\\text\{(.*?)\}", r"\1", s)
    s = s.replace("\\left", "").replace("\\right", "").replace("dfrac", "frac").replace("tfrac", "frac")
    s = s.rstrip(".")
    if re.fullmatch(r"-?\d+\.0+", s):
        s = s.split(".")[0]
    return s


def is_equiv(a: str | None, b: str | None) -> bool:
    if a is None or b is None:
        return False
    na, nb = normalize(a), normalize(b)
    if na == nb:
        return True
    try:
        return abs(float(na) - float(nb)) < 1e-6
    except ValueError:
        return False


class MathVerifier(BaseVerifier):
    def verify(self, response: str, answer: str) -> float:
        return 1.0 if is_equiv(last_boxed(response), answer) else 0.0
