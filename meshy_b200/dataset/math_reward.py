"""Rule-based math answer grading.

Three graders, matching what the reference's datasets use:

* :func:`math_reward` / :func:`grade_answer_verl` (MATH-style boxed answers; the reference's
  ``meshy/dataset/math_reward.py``, itself the DeepScaleR / Miles ``--rm-type math`` checker): the last
  ``\\boxed{}`` of the response is correct if it equals the ground truth after the Hendrycks MATH string
  normalisation (:func:`mathd_normalize`), or if the two are equal as SymPy expressions after a second,
  looser normalisation (:func:`sympy_normalize`, element-wise for tuples and intervals);
* :func:`dapo_compute_score` (the DAPO-Math-17k recipe, ``meshy/dataset/dapo_reward.py``, from VERL's
  ``math_dapo``): ``+1`` / ``-1``; strict mode compares the last box of the response's final 100 characters
  verbatim, the default (Minerva) mode compares the normalised ``Answer:`` line;
* :func:`gsm8k_reward`: the number after the last ``####``.

The normalisation steps and their substitution tables are the published ones (Hendrycks et al. MATH;
Lewkowycz et al. Minerva), since a grade is only comparable under the same rules; the code is this
package's. One difference: the reference turns LaTeX into text with ``pylatexenc`` before SymPy, which is
not installable here; :func:`latex_to_expr` is this package's own converter for the constructs that occur
in answers (fractions, roots, powers, products, constants, text wrappers).
"""

from __future__ import annotations

import re

# ───────────────────────────── boxed answers ─────────────────────────────


def _braced(text: str, start: int) -> tuple[str, int] | None:
    """Content of the brace group opening at ``text[start] == '{'`` and the index after its close."""
    if start >= len(text) or text[start] != "{":
        return None
    depth = 0
    for k in range(start, len(text)):
        c = text[k]
        if c == "{":
            depth += 1
        elif c == "}":
            depth -= 1
            if depth == 0:
                return text[start + 1:k], k + 1
    return None


def last_boxed(text: str) -> str | None:
    """Content of the last ``\\boxed{...}`` (or ``\\fbox{...}``) in ``text``; ``None`` if absent or unclosed."""
    at = text.rfind("\\boxed")
    if at < 0:
        at = text.rfind("\\fbox")
        if at < 0:
            return None
    brace = text.find("{", at)
    if brace < 0:
        return None
    got = _braced(text, brace)
    return got[0] if got else None


def _boxed_strict(text: str) -> str | None:
    """Content of the last ``\\boxed{`` group spelled exactly that way (DAPO's strict extraction)."""
    at = text.rfind("\\boxed{")
    if at < 0:
        return None
    got = _braced(text, at + len("\\boxed"))
    return got[0] if got else None


# ─────────────────────── Hendrycks MATH normalisation ───────────────────────


def _brace_fracs(s: str) -> str:
    """``\\frac12`` -> ``\\frac{1}{2}``, ``\\frac1{2}`` -> ``\\frac{1}{2}``."""
    head, *rest = s.split("\\frac")
    out = [head]
    for piece in rest:
        out.append("\\frac")
        if piece.startswith("{"):
            out.append(piece)
            continue
        if len(piece) < 2:
            return s
        a, b = piece[0], piece[1]
        out.append("{%s}%s" % (a, b + piece[2:]) if b == "{" else "{%s}{%s}%s" % (a, b, piece[2:]))
    return "".join(out)


def _slash_to_frac(s: str) -> str:
    parts = s.split("/")
    if len(parts) != 2:
        return s
    try:
        a, b = int(parts[0]), int(parts[1])
    except ValueError:
        return s
    return "\\frac{%d}{%d}" % (a, b) if s == "%d/%d" % (a, b) else s


def _brace_sqrt(s: str) -> str:
    if "\\sqrt" not in s:
        return s
    head, *rest = s.split("\\sqrt")
    out = [head]
    for piece in rest:
        out.append("\\sqrt" + piece if piece.startswith("{") else "\\sqrt{%s}%s" % (piece[:1], piece[1:]))
    return "".join(out)


def mathd_normalize(answer: str | None) -> str | None:
    """The MATH benchmark's answer string normalisation."""
    if answer is None:
        return None
    s = answer.strip()
    m = re.fullmatch(r"\\text\{(.+?)\}", s)
    if m:
        s = m.group(1).strip()
    try:
        for old, new in (("\n", ""), ("\\!", ""), ("\\\\", "\\"), ("tfrac", "frac"), ("dfrac", "frac"),
                         ("\\left", ""), ("\\right", ""), ("^{\\circ}", ""), ("^\\circ", ""), ("\\$", "")):
            s = s.replace(old, new)
        if "\\text{ " in s:  # trailing units
            pieces = s.split("\\text{ ")
            if len(pieces) != 2:
                return s
            s = pieces[0]
        s = s.replace("\\%", "").replace(" .", " 0.").replace("{.", "{0.")
        if not s:
            return s
        if s[0] == ".":
            s = "0" + s
        lhs_rhs = s.split("=")
        if len(lhs_rhs) == 2 and len(lhs_rhs[0]) <= 2:  # "x = 3" -> "3"
            s = lhs_rhs[1]
        s = _brace_sqrt(s).replace(" ", "")
        s = _brace_fracs(s)
        if s == "0.5":
            s = "\\frac{1}{2}"
        return _slash_to_frac(s)
    except IndexError:
        return answer


def grade_answer_mathd(given: str, truth: str) -> bool:
    return mathd_normalize(truth) == mathd_normalize(given)


# ─────────────────────── SymPy equivalence ───────────────────────

_UNITS = ("degree", "cm", "centimeter", "meter", "mile", "second", "minute", "hour", "day", "week", "month",
          "year", "foot", "feet", "inch", "yard")


def _replace_command(s: str, name: str, fn) -> str:
    """Replace ``\\name{a}{b}...`` (arity = fn's argument count) innermost-last by ``fn(a, b, ...)``."""
    import inspect

    arity = len(inspect.signature(fn).parameters)
    token = "\\" + name
    while True:
        at = s.find(token)
        if at < 0:
            return s
        pos = at + len(token)
        args = []
        for _ in range(arity):
            while pos < len(s) and s[pos] == " ":
                pos += 1
            got = _braced(s, pos)
            if got is None:  # single-character argument
                if pos >= len(s):
                    return s
                args.append(s[pos])
                pos += 1
            else:
                args.append(latex_to_expr(got[0]))
                pos = got[1]
        s = s[:at] + fn(*args) + s[pos:]


def latex_to_expr(s: str) -> str:
    """Answer-level LaTeX -> a SymPy-parsable expression string."""
    s = s.replace("\\left", "").replace("\\right", "").replace("\\!", "").replace("\\,", "").replace("\\;", "")
    s = s.replace("\\dfrac", "\\frac").replace("\\tfrac", "\\frac")
    for wrapper in ("text", "mathrm", "textbf", "mathbf", "operatorname"):
        s = _replace_command(s, wrapper, lambda a: a)
    s = _replace_command(s, "frac", lambda a, b: "((%s)/(%s))" % (a, b))
    m = re.search(r"\\sqrt\[([^\]]+)\]", s)
    while m:  # n-th roots
        rest = s[m.end():]
        got = _braced(rest, 0)
        if got is None:
            break
        s = s[:m.start()] + "((%s)**(1/(%s)))" % (latex_to_expr(got[0]), m.group(1)) + rest[got[1]:]
        m = re.search(r"\\sqrt\[([^\]]+)\]", s)
    s = _replace_command(s, "sqrt", lambda a: "sqrt(%s)" % a)
    for tex, plain in (("\\cdot", "*"), ("\\times", "*"), ("\\div", "/"), ("\\pi", "pi"), ("\\infty", "inf"),
                       ("\\cup", "U"), ("\\le", "<="), ("\\ge", ">=")):
        s = s.replace(tex, plain)
    s = re.sub(r"\^\{([^{}]*)\}", r"^(\1)", s)
    return s.strip()


def _drop_thousands(s: str) -> str:
    pat = re.compile(r"(\d),(\d\d\d)($|\D)")
    while True:
        t = pat.sub(r"\1\2\3", s)
        if t == s:
            return t
        s = t


def _as_int(s: str) -> int | None:
    try:
        v = float(_drop_thousands(s))
    except ValueError:
        return None
    return int(round(v)) if abs(v - round(v)) <= 1e-7 else None


def sympy_normalize(expr: str | None) -> str | None:
    """The looser normalisation applied before the SymPy comparison (units, words, LaTeX, case)."""
    if expr is None:
        return None
    m = re.fullmatch(r"\\text\{(.+?)\}", expr)
    if m:
        expr = m.group(1)
    expr = expr.replace("\\%", "%").replace("\\$", "$").replace("$", "").replace("%", "")
    expr = expr.replace(" or ", " , ").replace(" and ", " , ")
    for word, power in (("million", "6"), ("billion", "9"), ("trillion", "12")):
        expr = expr.replace(word, "*10^" + power)
    for unit in _UNITS:
        expr = re.sub(unit + r"(es)?(s)? *(\^[0-9]+)?", "", expr)
    expr = re.sub(r"\^ *\\circ", "", expr)
    if expr[:1] == "{" and expr[-1:] == "}":
        expr = expr[1:-1]
    expr = re.sub(r",\\! *", "", expr)
    try:
        f = float(expr)
        if abs(f - round(f)) <= 1e-7:
            expr = str(int(round(f)))
    except ValueError:
        pass
    if "\\" in expr:
        try:
            expr = latex_to_expr(expr)
        except Exception:  # noqa: BLE001 - leave unparsable LaTeX as it is
            pass
    expr = re.sub(r"- *", "-", expr)
    expr = re.sub(r"([0-9]) +([0-9])", r"\1+\2", expr)  # mixed numbers: "3 1/2" -> "3+1/2"
    expr = expr.replace(" ", "").replace("{", "").replace("}", "").lower()
    n = _as_int(expr)
    return str(n) if n is not None else expr


def _is_plain_fraction(e: str) -> bool:
    return re.fullmatch(r"-?[0-9]+.?/0*[1-9][0-9]*.?", e) is not None


def _safe_for_sympy(e: str) -> bool:
    letters = {c for c in e.replace("sqrt", "").replace("frac", "") if c.isalpha()}
    if len(letters) > 2:
        return False
    if "^{" in e or "^(" in e:
        return False
    return re.search(r"\^[0-9]+\^", e) is None and re.search(r"\^[0-9][0-9]+", e) is None


def sympy_equal(a: str, b: str) -> bool:
    """``a - b`` simplifies to 0 (guarded against expressions SymPy would take too long on)."""
    diff = "(%s)-(%s)" % (a, b)
    if not _safe_for_sympy(diff):
        return False
    try:
        import sympy
        from sympy.parsing import sympy_parser as P

        parsed = P.parse_expr(diff.replace("^", "**"),
                              transformations=P.standard_transformations + (P.implicit_multiplication_application,))
        return sympy.simplify(parsed) == 0
    except Exception:  # noqa: BLE001 - anything SymPy cannot handle is "not equal"
        return False


def _elements(e: str) -> list[str]:
    """Tuple / interval elements of a normalised answer (a plain answer is one element)."""
    e = _drop_thousands(e)
    if not e:
        return []
    brackets = "()[]"
    if len(e) > 2 and e[0] in brackets and e[-1] in brackets and not any(c in e[1:-1] for c in brackets):
        return [x.strip() for x in e[1:-1].split(",")]
    return [e]


def grade_answer_sympy(given: str, truth: str) -> bool:
    t, g = sympy_normalize(truth), sympy_normalize(given)
    if t is None:
        return False
    if t == g:
        return True
    if not g:
        return False
    te, ge = _elements(t), _elements(g)
    if len(te) > 1 and (t[0] != g[0] or t[-1] != g[-1]):  # open/closed bracket must agree
        return False
    if len(te) != len(ge):
        return False
    for x, y in zip(te, ge):
        if _is_plain_fraction(x) and _is_plain_fraction(y):
            ok = x == y
        elif (_as_int(x) is None) != (_as_int(y) is None):
            ok = False
        else:
            ok = sympy_equal(x, y)
        if not ok:
            return False
    return True


def grade_answer_verl(response: str, truth: object) -> bool:
    """The response's last boxed answer against the ground truth (boxed or plain)."""
    if not truth:
        return False
    t = str(truth)
    if "\\boxed" in t:
        t = last_boxed(t)
        if t is None:
            return False
    given = last_boxed(response) if "\\boxed" in response else None
    if given is None:
        return False
    return grade_answer_mathd(given, t) or grade_answer_sympy(given, t)


def math_reward(response: str, truth: object) -> float:
    return float(grade_answer_verl(response, truth))


# ─────────────────────── DAPO (VERL math_dapo) ───────────────────────

_MINERVA_SUBSTITUTIONS = (("an ", ""), ("a ", ""), (".$", "$"), ("\\$", ""), ("\\ ", ""), (" ", ""),
                          ("mbox", "text"), (",\\text{and}", ","), ("\\text{and}", ","), ("\\text{m}", "\\text{}"))
_MINERVA_REMOVED = ("square", "ways", "integers", "dollars", "mph", "inches", "hours", "km", "units", "\\ldots", "sue",
                    "points", "feet", "minutes", "digits", "cents", "degrees", "cm", "gm", "pounds", "meters",
                    "meals", "edges", "students", "childrentickets", "multiples", "\\text{s}", "\\text{.}",
                    "\\text{\ns}", "\\text{}^2", "\\text{}^3", "\\text{\n}", "\\text{}", "\\mathrm{th}", "^\\circ",
                    "^{\\circ}", "\\;", ",\\!", "{,}", '"', "\\dots")


def minerva_normalize(answer: str) -> str:
    """Minerva's final-answer normalisation (used by DAPO's non-strict mode)."""
    s = answer.split("=")[-1]
    for old, new in _MINERVA_SUBSTITUTIONS:
        s = s.replace(old, new)
    for junk in _MINERVA_REMOVED:
        s = s.replace(junk, "")
    s = re.sub(r"(.*?)(\$)(.*?)(\$)(.*)", "$\\3$", s)
    for cmd in ("text", "textbf", "overline"):
        s = re.sub(r"(\\%s\{)(.*?)(\})" % cmd, "\\2", s)
    s = re.sub(r"(\\boxed\{)(.*)(\})", "\\2", s)
    s = re.sub(r"(frac)([^{])(.)", "frac{\\2}{\\3}", s)
    s = re.sub(r"(sqrt)([^{])", "sqrt{\\2}", s)
    s = s.replace("$", "")
    if s.replace(",", "").isdigit():
        s = s.replace(",", "")
    return s.strip()


def dapo_compute_score(solution: str, ground_truth: str, strict_box_verify: bool = False) -> dict:
    """``{"score": +-1.0, "acc": bool, "pred": str | None}`` as the DAPO recipe scores a response."""
    tail = solution[-300:]
    if strict_box_verify:
        pred = _boxed_strict(tail[-100:])
        ok = pred == ground_truth
    else:
        found = re.findall(r"(?i)Answer\s*:\s*([^\n]+)", tail)
        pred = minerva_normalize(found[-1] if found else "[INVALID]")
        ok = pred == minerva_normalize(ground_truth)
    return {"score": 1.0 if ok else -1.0, "acc": ok, "pred": pred}


# ─────────────────────── compatibility helpers ───────────────────────


def normalize(ans: str) -> str:
    """Light answer-string normalisation (spaces, ``\\left``/``\\right``, ``\\text``, trailing period)."""
    s = re.sub(r"\\text\{([^}]*)\}", r"\1", ans.strip())
    for t in ("\\left", "\\right", "\\!", "\\,", "\\;", "$", " "):
        s = s.replace(t, "")
    return s.replace("dfrac", "frac").replace("tfrac", "frac").rstrip(".")


def boxed_reward(response: str, truth: str) -> float:
    """1.0 when the last boxed answer grades correct under :func:`grade_answer_verl`."""
    return math_reward(response, truth)


def gsm8k_answer(text: str) -> float | None:
    """The number after the first ``####`` of ``text`` (commas dropped), as the reference's GSM8K reads it."""
    m = re.search(r"####\s*(-?[\d,]+\.?\d*)", text)
    if m is None:
        return None
    try:
        return float(m.group(1).replace(",", ""))
    except ValueError:
        return None


def gsm8k_reward(response: str, truth) -> float:
    """1.0 when the response's ``####`` number equals the ground truth's (a number, or an answer string)."""
    pred = gsm8k_answer(response)
    want = truth if isinstance(truth, (int, float)) else gsm8k_answer(str(truth))
    if want is None and truth is not None and not isinstance(truth, (int, float)):
        try:
            want = float(str(truth).replace(",", ""))
        except ValueError:
            want = None
    return 1.0 if pred is not None and want is not None and pred == float(want) else 0.0


__all__ = ["boxed_reward", "dapo_compute_score", "grade_answer_mathd", "grade_answer_sympy", "grade_answer_verl",
           "gsm8k_answer", "gsm8k_reward", "last_boxed", "latex_to_expr", "math_reward", "mathd_normalize",
           "minerva_normalize", "normalize", "sympy_equal", "sympy_normalize"]
