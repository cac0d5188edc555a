"""Rule-based math answer checking (boxed-answer extraction + normalised compare).

Covers the reference's GSM8K ``####`` matcher and the MATH/DAPO strict-box
verifier (``meshy/dataset/gsm8k.py``, ``math.py``, ``dapo_reward.py``) with one
normaliser: strip spaces, ``\\left``/``\\right``, ``\\!``, trailing ``.``,
``\\text{..}`` wrappers, dollar signs, commas in integers; compare as exact
strings, then as numbers (fractions allowed).
"""

from __future__ import annotations

import re
from fractions import Fraction


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
    s = ans.strip()
    s = re.sub(r"\\text\{([^}]*)\}", r"\1", s)
    for t in ("\\left", "\\right", "\\!", "\\,", "\\;", "$", " "):
        s = s.replace(t, "")
    s = s.replace("dfrac", "frac").replace("tfrac", "frac")
    s = s.rstrip(".")
    if re.fullmatch(r"-?\d{1,3}(,\d{3})+", s):
        s = s.replace(",", "")
    return s


def _as_number(s: str):
    m = re.fullmatch(r"\\frac\{(-?\d+)\}\{(-?\d+)\}", s)
    try:
        if m:
            return Fraction(int(m.group(1)), int(m.group(2)))
        if re.fullmatch(r"-?\d+/\d+", s):
            a, b = s.split("/")
            return Fraction(int(a), int(b))
        return Fraction(s)
    except (ValueError, ZeroDivisionError):
        return None


def is_equiv(pred: str | None, truth: str | None) -> bool:
    if pred is None or truth is None:
        return False
    a, b = normalize(pred), normalize(str(truth))
    if a == b:
        return True
    x, y = _as_number(a), _as_number(b)
    return x is not None and y is not None and x == y


def _truth(truth) -> str | None:
    """The ground truth as an answer string: a boxed ground truth is unwrapped."""
    if truth is None:
        return None
    t = str(truth)
    return last_boxed(t) if "\\boxed" in t or "\\fbox" in t else t


def boxed_reward(response: str, truth: str) -> float:
    """1 when the response's last boxed answer equals the ground truth (strict form: ``2+2`` is not ``4``)."""
    return 1.0 if is_equiv(last_boxed(response), _truth(truth)) else 0.0


# names of the reference's math reward entry points (``meshy/dataset/math_reward.py``)
math_reward = boxed_reward


def grade_answer_verl(response: str, truth: str) -> bool:
    return boxed_reward(response, truth) == 1.0


def gsm8k_reward(response: str, truth: str) -> float:
    m = re.findall(r"####\s*([-\d,\.]+)", response)
    pred = m[-1] if m else last_boxed(response)
    t = str(truth).split("####")[-1].strip()
    return 1.0 if is_equiv(pred, t) else 0.0


__all__ = ["boxed_reward", "grade_answer_verl", "gsm8k_reward", "is_equiv", "last_boxed", "math_reward", "normalize"]
