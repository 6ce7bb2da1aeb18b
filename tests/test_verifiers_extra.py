"""DAPO / Minerva scoring and the sandboxed code executor (reference ``axrl/verifier``)."""

from axrl_b200.verifier.code_executor import check_assert_tests, check_io_tests, run_python
from axrl_b200.verifier.dapo import DapoVerifier, compute_score, minerva_correct, normalize_final_answer


def test_dapo_scores():
    assert compute_score("so the result is \\boxed{42}", "42") == 1.0
    assert compute_score("so the result is \\boxed{41}", "42") == 0.0
    assert compute_score("long reasoning...\nAnswer: $\\frac12$", "\\frac{1}{2}", strict_box_verify=False) == 1.0
    assert minerva_correct("Answer: 1,000 dollars", "1000")[0]
    assert normalize_final_answer("x = \\text{5 feet}") == "5"
    assert DapoVerifier().verify("\\boxed{7}", "7") == 1.0


def test_code_executor():
    ok, res = check_io_tests("print(sum(map(int, input().split())))", [("1 2", "3"), ("5 5", "10"), ("0 0", "1")])
    assert abs(ok - 2 / 3) < 1e-9 and res[2].status == "failed"
    assert run_python("while True: pass", timeout_s=0.5).status == "timeout"
    assert run_python("raise SystemExit(3)").status == "error"
    assert check_assert_tests("def f(x):\n    return x * 2", "assert f(3) == 6").passed
    assert not check_assert_tests("def f(x):\n    return x", "assert f(3) == 6").passed
