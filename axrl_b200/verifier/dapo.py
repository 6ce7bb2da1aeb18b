"""DAPO-style math reward: a strict boxed check on the tail of the response, or a Minerva-style
``Answer: ...`` extraction compared after normalisation.

Reference behaviour: ``axrl/verifier/dapo_utils.py:6-266`` (DAPO / Minerva scoring used by the
DAPO17k recipes): only the last 300 characters are inspected; strict mode looks for the last
``\\boxed{...}`` in the final 100 characters and compares it verbatim; Minerva mode takes the last
``Answer:`` line and compares normalised strings.  Reward is 1.0 or 0.0.
"""

from __future__ import annotations

import re

from axrl_b200.verifier.base_verifier import BaseVerifier
from axrl_b200.verifier.math_reward import last_boxed

_UNITS = ("square", "ways", "integers", "dollars", "mph", "inches", "ft", "hours", "km", "units", "\\ldots", "sue", "points",
          "feet", "minutes", "digits", "cents", "degrees", "cm", "gm", "pounds", "meters", "meals", "edges", "students",
          "childrentickets", "multiples", "\\text{s}", "\\text{.}", "\\text{\ns}", "\\text{}^2", "\\text{}^3", "\\text{\n}", "\\text{}",
          r"\mathrm{th}", r"^\circ", r"^{\circ}", r"\;", r",\!", "{,}", '"', "\\dots")


def normalize_final_answer(ans: str) -> str:
    """Canonical form of a final answer string (Minerva-style)."""
    s = ans.split("=")[-1]
    for a, b in (("an ", ""), ("a ", ""), (".$", "$"), ("\\$", ""), (r"\ ", ""), (" ", ""), ("mbox", "text"),
                 (",\\text{and}", ","), ("\\text{and}", ","), ("\\text{m}", "\\text{}")):
        s = s.replace(a, b)
    for u in _UNITS:
        s = s.replace(u, "")
    s = re.sub(r"(.*?)(\$)(.*?)(\$)(.*)", "$\\3$", s)          # keep the last $...$ span
    s = re.sub(r"(\\text\{)(.*?)(\})", "\\2", s)
    s = re.sub(r"(\\textbf\{)(.*?)(\})", "\\2", s)
    s = re.sub(r"(\\overline\{)(.*?)(\})", "\\2", s)
    s = re.sub(r"(\\boxed\{)(.*)(\})", "\\2", s)
    s = re.sub(r"(frac)([^{])(.)", "frac{\\2}{\\3}", s)         # \frac12 -> \frac{1}{2}
    s = re.sub(r"(sqrt)([^{])", "sqrt{\\2}", s)                  # \sqrt2 -> \sqrt{2}
    s = s.replace("$", "")
    if s.replace(",", "").isdigit():                             # 1,000 -> 1000
        s = s.replace(",", "")
    return s.strip()


def strict_box_correct(response: str, gt: str) -> tuple[bool, str | None]:
    inner = last_boxed(response[-100:])
    return inner == gt, inner


def minerva_correct(response: str, gt: str, gt_boxed: bool = False) -> tuple[bool, str]:
    found = re.findall(r"(?i)Answer\s*:\s*([^\n]+)", response)
    pred = normalize_final_answer(found[-1] if found else "[INVALID]")
    if gt_boxed:
        inner = last_boxed(gt)
        assert inner is not None, "ground truth has no boxed answer"
        gt = inner
    return pred == normalize_final_answer(gt), pred


def compute_score(response: str, ground_truth: str, strict_box_verify: bool = True) -> float:
    tail = response[-300:]
    ok = strict_box_correct(tail, ground_truth)[0] if strict_box_verify else minerva_correct(tail, ground_truth)[0]
    return 1.0 if ok else 0.0


class DapoVerifier(BaseVerifier):
    def __init__(self, strict_box_verify: bool = True) -> None:
        self.strict = strict_box_verify

    def verify(self, response: str, answer: str) -> float:
        return compute_score(response, answer, self.strict)


class HfMathVerifier(BaseVerifier):
    """Symbolic equivalence through the ``math_verify`` package when installed (reference
    ``axrl/verifier/hf_math_verifier.py:14``); otherwise the boxed-answer normaliser."""

    def __init__(self) -> None:
        try:
            import math_verify  # noqa: F401

            self.mv = math_verify
        except ImportError:
            self.mv = None

    def verify(self, response: str, answer: str) -> float:
        if self.mv is not None:
            gold, pred = self.mv.parse(answer), self.mv.parse(response)
            return 1.0 if self.mv.verify(gold, pred) else 0.0
        from axrl_b200.verifier.math_reward import MathVerifier

        return MathVerifier().verify(response, answer)
