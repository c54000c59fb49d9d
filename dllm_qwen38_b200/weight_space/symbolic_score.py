"""Boxed-answer scorer for MATH-style runs (the reference's `tools/weight-space/symbolic_score.py:13-79`
role).

Two profiles. When math-verify and its parser stack are installed at the versions the reference
pins (math-verify 0.9.0, latex2sympy2-extended 1.11.0, antlr4 4.13.2, sympy 1.14.0), the answer is
graded by math-verify with the reference's settings (boxed extraction first, no fallback, strict
verification, 12-digit float rounding, 5 s parse / verify limits; main thread only) - profile
`boxed-math-verify-0.9.0`, so grades agree with the reference's. Otherwise the profile below, our
own, is used:

score(gold, content, thinking_open=False) -> {"profile", "status", "correct"}:
  * text inside <think>...</think> is ignored (an unfinished or malformed think block is a status,
    not a crash); `thinking_open` says the content starts inside a think block;
  * the LAST \\boxed{...} outside thinking is the answer (braces balanced, escaped braces skipped);
  * gold and answer are compared as exact rationals when both parse as numbers (integers,
    decimals, a/b, \\frac{a}{b} / \\dfrac / \\tfrac, signs, thousands separators, a trailing
    unit-free `^\\circ` or `\\%`); otherwise as normalised LaTeX strings (spacing, \\left / \\right,
    \\!, \\, and \\text{} wrappers removed);
  * status is "scored" with correct True/False, a parse status with correct False, or
    "grader_unavailable" with correct None when the gold itself cannot be read.
No raw answer text is returned.
"""

from __future__ import annotations

import re
from fractions import Fraction

PROFILE_OWN = "boxed-rational-or-normalised-latex/v1"
PROFILE_MV = "boxed-math-verify-0.9.0"
PINNED = {"math-verify": "0.9.0", "latex2sympy2-extended": "1.11.0", "antlr4-python3-runtime": "4.13.2",
          "sympy": "1.14.0"}


def _pinned_math_verify() -> bool:
    import importlib.metadata as md

    try:
        return all(md.version(k) == v for k, v in PINNED.items())
    except md.PackageNotFoundError:
        return False


USE_MV = _pinned_math_verify()
PROFILE = PROFILE_MV if USE_MV else PROFILE_OWN
MAX_PRED = 65536
MAX_GOLD = 4096


def outside_thinking(text: str, thinking_open: bool = False) -> str:
    inside = bool(thinking_open)
    out, pos = [], 0
    for m in re.finditer(r"</?think>", text):
        if not inside:
            out.append(text[pos:m.start()])
        if m.group() == "<think>":
            if inside:
                raise ValueError("nested_thinking")
            inside = True
        else:
            if not inside:
                raise ValueError("unmatched_thinking_close")
            inside = False
        pos = m.end()
    if inside:
        raise ValueError("unfinished_thinking")
    out.append(text[pos:])
    return "".join(out)


def last_box(text: str) -> str:
    """Content of the last \\boxed{...} (without the wrapper)."""
    found, i = None, 0
    pat = re.compile(r"\\boxed\s*\{")
    while True:
        m = pat.search(text, i)
        if m is None:
            break
        # an escaped backslash before \boxed means it is literal text
        bs, j = 0, m.start() - 1
        while j >= 0 and text[j] == "\\":
            bs, j = bs + 1, j - 1
        if bs % 2:
            i = m.end()
            continue
        depth, k = 1, m.end()
        while k < len(text) and depth:
            c = text[k]
            if c == "\\" and k + 1 < len(text):
                k += 2
                continue
            depth += (c == "{") - (c == "}")
            k += 1
        if depth:
            raise ValueError("unfinished_box")
        found, i = text[m.end():k - 1], k
    if found is None:
        raise ValueError("missing_box")
    return found


def _strip(s: str) -> str:
    s = s.strip().strip("$").strip()
    s = re.sub(r"\\text\s*\{([^{}]*)\}", r"\1", s)
    s = re.sub(r"\\(left|right|!|,|;|:)", "", s)
    s = s.replace("\\dfrac", "\\frac").replace("\\tfrac", "\\frac")
    s = re.sub(r"\^\s*\{?\\circ\}?", "", s).replace("\\%", "").replace("%", "")
    s = re.sub(r"\s+", "", s)
    return s.rstrip(".")


def as_rational(s: str):
    s = _strip(s)
    sign = 1
    while s[:1] in "+-" and s:
        sign, s = (-sign if s[0] == "-" else sign), s[1:]
    m = re.fullmatch(r"\\frac\{([^{}]+)\}\{([^{}]+)\}", s) or re.fullmatch(r"\\frac(\d)(\d)", s)
    if m:
        a, b = as_rational(m.group(1)), as_rational(m.group(2))
        if a is None or b is None or b == 0:
            return None
        return sign * a / b
    m = re.fullmatch(r"([^/]+)/([^/]+)", s)
    if m:
        a, b = as_rational(m.group(1)), as_rational(m.group(2))
        if a is None or b is None or b == 0:
            return None
        return sign * a / b
    if re.fullmatch(r"\d{1,3}(,\d{3})+(\.\d+)?", s):
        s = s.replace(",", "")
    if re.fullmatch(r"\d+(\.\d*)?|\.\d+", s):
        return sign * Fraction(s)
    return None


def score(gold: str, content: str, *, thinking_open: bool = False) -> dict:
    if not isinstance(gold, str) or not gold or len(gold.encode()) > MAX_GOLD:
        raise ValueError("invalid_reference_size")
    if len(content.encode()) > MAX_PRED:
        return {"profile": PROFILE, "status": "prediction_too_long", "correct": False}
    if not _strip(gold):
        return {"profile": PROFILE, "status": "grader_unavailable", "correct": None}
    try:
        ans = last_box(outside_thinking(content, thinking_open))
    except ValueError as e:
        return {"profile": PROFILE, "status": str(e), "correct": False}
    if not _strip(ans):
        return {"profile": PROFILE, "status": "prediction_unparsed", "correct": False}
    if USE_MV:
        return _score_math_verify(gold, ans)
    g, a = as_rational(gold), as_rational(ans)
    ok = (g == a) if (g is not None and a is not None) else (_strip(gold) == _strip(ans))
    return {"profile": PROFILE, "status": "scored", "correct": bool(ok)}


def _score_math_verify(gold: str, ans: str) -> dict:
    import threading

    if threading.current_thread() is not threading.main_thread():
        raise RuntimeError("math-verify grading uses POSIX alarms: main thread only")
    from math_verify import LatexExtractionConfig, parse, verify

    cfg = [LatexExtractionConfig(boxed_match_priority=0)]

    def rd(text):
        return parse(text, extraction_config=cfg, fallback_mode="no_fallback", extraction_mode="first_match",
                     parsing_timeout=5, raise_on_error=True)

    try:
        ref = rd("\\boxed{" + gold + "}")
    except Exception:  # noqa: BLE001
        return {"profile": PROFILE, "status": "grader_unavailable", "correct": None}
    if not ref:
        return {"profile": PROFILE, "status": "grader_unavailable", "correct": None}
    try:
        pred = rd("\\boxed{" + ans + "}")
        if not pred:
            return {"profile": PROFILE, "status": "prediction_unparsed", "correct": False}
        ok = verify(ref, pred, float_rounding=12, numeric_precision=30, strict=True, allow_set_relation_comp=False,
                    timeout_seconds=5, raise_on_error=True)
    except Exception as e:  # noqa: BLE001
        return {"profile": PROFILE, "status": "grader_unavailable", "correct": None, "error_type": type(e).__name__}
    return {"profile": PROFILE, "status": "scored", "correct": bool(ok)}
