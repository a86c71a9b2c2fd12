"""Rule-based rewards for GRPO: math answers, response format, code tests, length, thinking.

Reference: ``mamformer/rewards.py`` (``math_reward`` 94-160, ``format_reward`` 163-209,
``code_reward`` 212-262 with the sandbox of 288-420, ``length_penalty`` 423-478,
``thinking_quality_reward`` 481-566, ``RewardCalculator`` 569-674).  The score tables are the
reference's so that rewards (and therefore advantages) agree between the two frameworks:

* math: 1.0 when the last ``\\boxed{...}`` equals the ground truth (numerically within 1e-4
  relative / 1e-6 absolute, or as a case- and space-insensitive string); 0.3 for a wrong answer
  in ``<think>...</think><answer>...</answer>`` form; else 0;
* format: 1.0 think-then-answer with content, 0.7 reversed, 0.5 only one part, 0;
* code: fraction of test cases whose call returns the expected string, each run in a separate
  interpreter with dangerous builtins removed, imports / dunder traversal rejected up front,
  a 512 MB address-space limit and a timeout;
* length (words): linear ramp to 1 at ``target``, linear decay to 0.5 at ``max``, 0.5 beyond;
* thinking: structure 0.4 / 0.25 / 0.1, substance 0.3 / 0.2 / 0.05, order 0.2 / 0.1,
  multi-path bonus 0.1, capped at 1.
"""

from __future__ import annotations

import json
import os
import re
import subprocess
import sys
import tempfile
from typing import Callable, Dict, List, Optional

# ---- answers -------------------------------------------------------------------------------
_BOXED = re.compile(r"\\boxed\{")


def extract_boxed(text: str) -> List[str]:
    """Contents of every ``\\boxed{...}`` (nested braces balanced)."""
    out = []
    for m in _BOXED.finditer(text):
        depth, j = 1, m.end()
        while j < len(text) and depth:
            depth += {"{": 1, "}": -1}.get(text[j], 0)
            j += 1
        if depth == 0:
            out.append(text[m.end():j - 1])
    return out


_extract_boxed = extract_boxed


def parse_number(s: str) -> Optional[float]:
    """A number out of an answer string: fractions, scientific notation, LaTeX wrappers,
    thousands separators; the first number found otherwise."""
    if not s:
        return None
    t = s.strip()
    for tok in (r"\text", r"\mathrm"):
        t = t.replace(tok, "")
    t = re.sub(r"[{}$\\, ]", "", t)
    m = re.fullmatch(r"(-?\d+)/(-?\d+)", t)
    if m:
        den = float(m.group(2))
        return None if den == 0 else float(m.group(1)) / den
    if re.fullmatch(r"-?\d+\.?\d*[eE]-?\d+", t):
        try:
            return float(t)
        except ValueError:
            pass
    m = re.search(r"-?\d+\.?\d*", t)
    return float(m.group()) if m else None


_extract_numeric = parse_number


def _tagged(response: str, tag: str):
    return re.search(rf"<{tag}>(.*?)</{tag}>", response, re.DOTALL)


def math_reward(response: str, ground_truth: str) -> float:
    boxes = extract_boxed(response)
    if not boxes:
        return 0.0
    got, want = boxes[-1].strip(), ground_truth.strip()
    a, b = parse_number(got), parse_number(want)
    if a is not None and b is not None:
        if b == 0:
            if abs(a) < 1e-6:
                return 1.0
        elif abs(a - b) / max(abs(b), 1e-8) < 1e-4 or abs(a - b) < 1e-6:
            return 1.0
    if got.lower().replace(" ", "") == want.lower().replace(" ", ""):
        return 1.0
    return 0.3 if (_tagged(response, "think") and _tagged(response, "answer")) else 0.0


def format_reward(response: str) -> float:
    th, an = _tagged(response, "think"), _tagged(response, "answer")
    ok_t = th is not None and th.group(1).strip() != ""
    ok_a = an is not None and an.group(1).strip() != ""
    if ok_t and ok_a:
        return 1.0 if th.end() <= an.start() else 0.7
    return 0.5 if (ok_t or ok_a) else 0.0


# ---- code --------------------------------------------------------------------------------------
def extract_code(response: str) -> Optional[str]:
    """Last ```python block, else last fenced block, else the bare ``def`` blocks."""
    for pat in (r"```python\s*\n(.*?)```", r"```(?:\w*)?\s*\n(.*?)```"):
        blocks = re.findall(pat, response, re.DOTALL)
        if blocks:
            return blocks[-1].strip()
    defs = re.findall(r"(def\s+\w+\s*\([^)]*\).*?)(?:\n\n|\Z)", response, re.DOTALL)
    return "\n".join(defs) if defs else None


_extract_code = extract_code

_FORBIDDEN_CODE = [
    (r"__import__", "__import__"), (r"\bopen\s*\(", "open()"), (r"\beval\s*\(", "eval()"),
    (r"\bexec\s*\(", "exec()"), (r"\bcompile\s*\(", "compile()"), (r"\bglobals\s*\(\s*\)", "globals()"),
    (r"\blocals\s*\(\s*\)", "locals()"), (r"\bgetattr\s*\(", "getattr()"), (r"__builtins__", "__builtins__"),
    (r"__class__\s*\.", "__class__ traversal"), (r"__bases__", "__bases__"),
    (r"__subclasses__\s*\(\s*\)", "__subclasses__()"), (r"__globals__", "__globals__"),
    (r"\b(?:import|from)\s+\w+", "import statement"), (r"breakpoint\s*\(", "breakpoint()"),
    (r"copyright|credits|license", "interactive help builtins"),
]
_FORBIDDEN_INPUT = ("__import__", "os.system", "subprocess", "eval(", "exec(", "open(", "rm -", "shutil",
                    "import ", "compile(")
_REMOVED_BUILTINS = ["__import__", "open", "eval", "exec", "compile", "globals", "locals", "vars", "dir",
                     "getattr", "setattr", "delattr", "hasattr", "breakpoint", "input", "copyright",
                     "credits", "license", "help"]


def _scan_user_code(code: str) -> Optional[str]:
    for pat, what in _FORBIDDEN_CODE:
        if re.search(pat, code):
            return f"forbidden in user code: {what}"
    return None


def _is_safe_test_input(s: str) -> bool:
    low = s.lower()
    return not any(d in low for d in _FORBIDDEN_INPUT)


_HARNESS = """import sys, json, builtins
_args = json.loads(sys.argv[1]); _want = json.loads(sys.argv[2])
for _n in {removed!r}:
    builtins.__dict__.pop(_n, None)
    if isinstance(__builtins__, dict):
        __builtins__.pop(_n, None)
{code}
try:
    _got = {fn}(*_args) if isinstance(_args, list) else {fn}(_args)
    print("PASS" if str(_got).strip() == str(_want).strip() else "FAIL")
except Exception:
    print("FAIL")
"""


def _limit_memory():
    try:
        import resource
        lim = 512 * 1024 * 1024
        resource.setrlimit(resource.RLIMIT_AS, (lim, lim))
    except (ImportError, ValueError, OSError):
        pass


def _json_or_text(s: str):
    if not s.strip():
        return ""
    try:
        return json.loads(s)
    except (json.JSONDecodeError, ValueError):
        return s


def run_test_case(code: str, function_name: str, test_input: str, expected_output: str, timeout: int = 30) -> bool:
    if not re.fullmatch(r"[A-Za-z_][A-Za-z0-9_]*", function_name):
        return False
    if _scan_user_code(code) is not None or not _is_safe_test_input(test_input):
        return False
    script = _HARNESS.format(removed=_REMOVED_BUILTINS, code=code, fn=function_name)
    try:
        res = subprocess.run([sys.executable, "-I", "-c", script, json.dumps(_json_or_text(test_input)),
                              json.dumps(_json_or_text(expected_output) if expected_output.strip() else expected_output)],
                             capture_output=True, text=True, timeout=timeout, cwd=tempfile.gettempdir(),
                             preexec_fn=_limit_memory if os.name == "posix" else None)
    except Exception:
        return False
    return "PASS" in res.stdout and "FAIL" not in res.stdout


_run_single_test = run_test_case


def code_reward(response: str, test_cases: List[dict], function_name: str = "solution", timeout: int = 30) -> float:
    if not test_cases:
        return 0.0
    code = extract_code(response)
    if code is None:
        return 0.0
    ok = sum(run_test_case(code, tc.get("function", function_name), tc.get("input", ""),
                           tc.get("expected_output", ""), timeout) for tc in test_cases)
    return ok / len(test_cases)


# ---- length and thinking -----------------------------------------------------------------------
def length_penalty(response: str, min_words: int = 50, max_words: int = 4096, target_words: int = 512,
                   min_tokens: Optional[int] = None, max_tokens: Optional[int] = None,
                   target_tokens: Optional[int] = None) -> float:
    lo = min_words if min_tokens is None else min_tokens
    hi = max_words if max_tokens is None else max_tokens
    tgt = target_words if target_tokens is None else target_tokens
    n = len(response.split())
    if n <= lo:
        return n / max(lo, 1)
    if n <= tgt:
        return lo / tgt + (1.0 - lo / tgt) * (n - lo) / (tgt - lo)
    if n <= hi:
        return 1.0 - 0.5 * (n - tgt) / (hi - tgt)
    return 0.5


_THINK_OPEN = r"<\|think_start\|>|<think_start>|<think>|<thinking>"
_THINK_CLOSE = r"<\|think_end\|>|<think_end>|</think>|</thinking>"
_ANSWER_OPEN = r"<\|answer_start\|>|<answer_start>|<answer>"
_THINK_BODIES = (r"<\|think_start\|>(.*?)<\|think_end\|>", r"<think_start>(.*?)<think_end>",
                 r"<think>(.*?)</think>", r"<thinking>(.*?)</thinking>")


def thinking_quality_reward(response: str) -> float:
    flags = re.IGNORECASE
    o = re.search(_THINK_OPEN, response, flags) is not None
    c = re.search(_THINK_CLOSE, response, flags) is not None
    a = re.search(_ANSWER_OPEN, response, flags) is not None
    score = 0.4 if (o and c and a) else 0.25 if (o and a) else 0.1 if o else 0.0
    for pat in _THINK_BODIES:
        m = re.search(pat, response, re.DOTALL | flags)
        if m:
            n = len(m.group(1).strip())
            score += 0.3 if n > 100 else 0.2 if n > 20 else 0.05
            break
    if o and a:
        low = response.lower()
        tp, ap = low.find("<think"), low.find("<answer")
        if tp >= 0 and ap >= 0:
            score += 0.2 if tp < ap else 0.1
    if len(re.findall(r"<\|think_start\|>|<think_start>|<think>", response, flags)) > 1:
        score += 0.1
    return min(score, 1.0)


# ---- dispatch ----------------------------------------------------------------------------------
class RewardCalculator:
    _DISPATCH: Dict[str, Callable[..., float]] = {
        "math": math_reward, "format": format_reward, "code": code_reward, "length": length_penalty,
        "thinking": thinking_quality_reward,
    }

    def compute(self, response: str, reward_type: str = "format", **kwargs) -> float:
        if reward_type == "combined":
            return self._combined_reward(response, **kwargs)
        fn = self._DISPATCH.get(reward_type)
        if fn is None:
            raise ValueError(f"Unknown reward_type '{reward_type}'. Available: {list(self._DISPATCH)} + 'combined'")
        return fn(response, **kwargs)

    def _combined_reward(self, response: str, **kwargs) -> float:
        weights = kwargs.pop("reward_weights", None)
        if weights is None:
            raise ValueError("'combined' reward type requires 'reward_weights' dict")
        tot = wsum = 0.0
        for kind, w in weights.items():
            fn = self._DISPATCH.get(kind)
            if fn is None:
                continue
            extra = kwargs.pop(kind, {})
            if not isinstance(extra, dict):
                raise TypeError(f"Expected dict for reward type '{kind}' kwargs, got {type(extra).__name__}")
            tot += w * fn(response, **extra)
            wsum += w
        return tot / wsum if wsum else 0.0

    def batch(self, responses: List[str], reward_type: str = "format", per_item: Optional[List[dict]] = None,
              **kwargs) -> List[float]:
        """Scores for a batch (``per_item[i]`` adds keyword arguments for response i)."""
        out = []
        for i, r in enumerate(responses):
            kw = dict(kwargs)
            if per_item is not None:
                kw.update(per_item[i])
            out.append(self.compute(r, reward_type, **kw))
        return out
