"""Math graders (CPU): the boxed-answer checker with string normalisation and SymPy equivalence, DAPO's
+-1 scorer in strict and Minerva modes, the GSM8K ``####`` match, and the S9 / DAPO / GSM8K record
formats of the datasets."""

import json

import pytest

from meshy_b200.dataset.math_reward import (dapo_compute_score, grade_answer_verl, gsm8k_reward, last_boxed,
                                            latex_to_expr, math_reward, mathd_normalize, minerva_normalize,
                                            sympy_normalize)


@pytest.mark.parametrize(("response", "truth", "expected"), [
    (r"\boxed{42}", "42", 1.0),
    (r"\boxed{wrong}", "42", 0.0),
    ("42", "42", 0.0),                                      # no boxed answer
    (r"first \boxed{0}, finally \boxed{42}", "42", 1.0),     # the last box counts
    (r"\boxed{\frac{1}{2}}", "0.5", 1.0),                   # string normalisation: 0.5 -> \frac{1}{2}
    (r"\boxed{\dfrac{3}{4}}", "3/4", 1.0),                  # a/b -> \frac{a}{b}
    (r"\boxed{2+2}", "4", 0.0),                             # an integer truth needs an integer answer
    (r"\boxed{2\cdot x}", "x+x", 1.0),                       # equal under SymPy
    (r"\boxed{x+1}", "1+x", 1.0),
    (r"\boxed{\frac{\sqrt{2}}{2}}", r"\frac{1}{\sqrt{2}}", 1.0),
    (r"\boxed{2x}", "x+x", 1.0),
    (r"\boxed{3}", "3.0", 1.0),
    (r"\boxed{42}", r"\boxed{42}", 1.0),                   # boxed ground truth
    (r"\boxed{42}", "", 0.0),
    (r"\boxed{1,000}", "1000", 1.0),
    (r"\boxed{10^{\circ}}", "10", 1.0),
    (r"\boxed{\text{(B)}}", "(B)", 1.0),
    (r"\boxed{(1, 2)}", "(1,2)", 1.0),                      # tuples element-wise
    (r"\boxed{[1, 2)}", "(1,2)", 0.0),                      # interval ends must agree
    (r"\boxed{1/2}", "2/4", 0.0),                           # plain fractions compare verbatim
    (r"\boxed{x = 5}", "5", 1.0),
])
def test_math_reward(response, truth, expected):
    assert math_reward(response, truth) == expected
    assert grade_answer_verl(response, truth) == (expected == 1.0)


def test_normalisers():
    assert last_boxed(r"a \boxed{\frac{1}{\sqrt{2}}} b") == r"\frac{1}{\sqrt{2}}"
    assert last_boxed(r"\boxed{unclosed") is None
    assert mathd_normalize(r"\frac12") == r"\frac{1}{2}"
    assert mathd_normalize(r"\sqrt2") == r"\sqrt{2}"
    assert mathd_normalize("5\\%") == "5"
    assert sympy_normalize("3 million") == "3*10^6"
    assert sympy_normalize("12 cm") == "12"
    assert latex_to_expr(r"\frac{a}{\sqrt{b}}") == "((a)/(sqrt(b)))"
    assert minerva_normalize(r"x = \$1,000") == "1000"


def test_dapo_score():
    assert dapo_compute_score(r"... so \boxed{7}", "7", strict_box_verify=True) == {"score": 1.0, "acc": True,
                                                                                     "pred": "7"}
    assert dapo_compute_score(r"\boxed{7.0}", "7", strict_box_verify=True)["score"] == -1.0  # verbatim only
    assert dapo_compute_score("x" * 400 + r"\boxed{7}", "7", strict_box_verify=True)["score"] == 1.0
    assert dapo_compute_score(r"\boxed{7}" + " " * 120, "7", strict_box_verify=True)["score"] == -1.0  # last 100
    assert dapo_compute_score("work...\nAnswer: 1,000 dollars", "1000")["score"] == 1.0
    assert dapo_compute_score("no answer line", "3")["score"] == -1.0


@pytest.mark.parametrize(("response", "truth", "expected"), [
    ("so the total is #### 72", "Natalia sold 48/2 = 24 ...\n#### 72", 1.0),
    ("#### 1,234", "#### 1234", 1.0),
    ("#### 1234", 1234.0, 1.0),
    (r"answer \boxed{18}", "#### 18", 0.0),   # only the #### form counts
    ("#### 5 then #### 7", "#### 7", 0.0),     # the first #### is the answer
    ("#### 8", "#### 7", 0.0),
])
def test_gsm8k_reward(response, truth, expected):
    assert gsm8k_reward(response, truth) == expected


class _Builder:
    """Stand-in builder: one token per character of every message."""

    def build_sample(self, messages):
        from meshy_b200.utils.sample import Sample

        s = Sample(messages=list(messages))
        s.extend([1] * sum(len(m["content"]) for m in messages), trained=False)
        return s


def test_dataset_record_formats(tmp_path):
    from meshy_b200.dataset.math import GSM8K, MATH, S9Math

    s9 = tmp_path / "s9.jsonl"
    s9.write_text(json.dumps({"prompt": [{"role": "user", "content": "1+1?"}], "label": "2"}) + "\n")
    ds = S9Math(batch_size=1, path=str(s9))
    sample = ds.next_batch(_Builder())[0]
    assert sample.ground_truth == "2" and sample.messages[0]["content"] == "1+1?"
    sample.messages.append({"role": "assistant", "content": r"\boxed{2}"})
    assert S9Math.reward(sample) == 1.0
    bad = tmp_path / "bad.jsonl"
    bad.write_text(json.dumps({"prompt": "text"}) + "\n")
    with pytest.raises(ValueError):
        S9Math(batch_size=1, path=str(bad))
    with pytest.raises(ValueError):
        S9Math(batch_size=1, path=str(s9), prompt_max_tokens=2).next_batch(_Builder())

    dapo = tmp_path / "dapo.jsonl"
    dapo.write_text(json.dumps({"prompt": [{"role": "user", "content": "Find x."}],
                                "reward_model": {"ground_truth": "34"}}) + "\n")
    m = MATH(batch_size=1, path=str(dapo)).next_batch(_Builder())[0]
    assert m.ground_truth == "34" and m.messages[0]["content"].startswith("Find x.")
    m.messages.append({"role": "assistant", "content": r"\boxed{34}"})
    assert MATH.reward(m) == 1.0
    m.messages[-1]["content"] = r"\boxed{35}"
    assert MATH.reward(m) == -1.0

    gsm = tmp_path / "gsm.jsonl"
    gsm.write_text(json.dumps({"question": "How many?", "answer": "steps\n#### 1,200"}) + "\n")
    g = GSM8K(batch_size=1, path=str(gsm)).next_batch(_Builder())[0]
    assert g.ground_truth == 1200.0 and g.messages[0]["role"] == "system"
    g.messages.append({"role": "assistant", "content": "#### 1200"})
    assert GSM8K.reward(g) == 1.0
