"""Rule-based math rewards: the last boxed answer against the ground truth, strict form (same cases as the
reference's reward behaviour: nested boxes, fractions vs decimals, boxed ground truths, unboxed responses),
plus the GSM8K ``####`` matcher."""

import pytest

from meshy_b200.dataset.math_reward import grade_answer_verl, gsm8k_reward, last_boxed, math_reward, normalize


@pytest.mark.parametrize(("response", "truth", "expected"), [
    (r"\boxed{42}", "42", 1.0),
    (r"\boxed{wrong}", "42", 0.0),
    ("42", "42", 0.0),                                   # no boxed answer
    (r"first \boxed{0}, finally \boxed{42}", "42", 1.0),  # the last box counts
    (r"\boxed{\frac{1}{2}}", "0.5", 1.0),
    (r"\boxed{\dfrac{3}{4}}", "3/4", 1.0),
    (r"\boxed{2+2}", "4", 0.0),                         # no algebraic simplification
    (r"\boxed{42}", r"\boxed{42}", 1.0),                # boxed ground truth
    (r"\boxed{42}", "", 0.0),
    (r"\boxed{1,000}", "1000", 1.0),
    (r"\boxed{\text{(B)}}", "(B)", 1.0),
    (r"\boxed{x^{2}}", "x^{2}", 1.0),
])
def test_math_reward(response, truth, expected):
    assert math_reward(response, truth) == expected
    assert grade_answer_verl(response, truth) == (expected == 1.0)


def test_helpers():
    assert last_boxed(r"a \boxed{\frac{1}{\sqrt{2}}} b") == r"\frac{1}{\sqrt{2}}"
    assert last_boxed(r"\boxed{unclosed") is None
    assert normalize(r" \left( 3 \right) .") == "(3)"


@pytest.mark.parametrize(("response", "truth", "expected"), [
    ("so the total is #### 72", "Natalia sold 48/2 = 24 ...\n#### 72", 1.0),
    ("#### 1,234", "#### 1234", 1.0),
    (r"answer \boxed{18}", "#### 18", 1.0),
    ("#### 5 then #### 7", "#### 7", 1.0),
    ("#### 8", "#### 7", 0.0),
])
def test_gsm8k_reward(response, truth, expected):
    assert gsm8k_reward(response, truth) == expected
