"""Pre-training data curation: read, classify by domain, score quality, near-deduplicate, mix.

Reference: ``scripts/data_pipeline.py`` (``DataMixConfig`` 53-75, ``DomainClassifier`` 77-186,
``QualityScorer`` 188-310, ``Deduplicator`` 313-427 (MinHash + LSH bands), ``ContentFilter``
429-494, ``DataMixer`` 496-566, ``MultiFormatReader`` 568-890, ``DataPipeline`` 892-1043) and
``configs/data_mix.yaml`` (domain weights, length / quality / dedup thresholds, seed), whose keys
are read unchanged.  The heuristics here are this module's own: domain scores are densities of
domain marker patterns, quality is a weighted mix of length, n-gram repetition, lexical
diversity and paragraph structure, near-duplicates are found with 128 MinHash permutations in
16 LSH bands and confirmed with the estimated Jaccard similarity.
"""

from __future__ import annotations

import csv
import hashlib
import html
import json
import math
import os
import random
import re
from collections import Counter, defaultdict
from dataclasses import dataclass, field
from typing import Dict, Iterator, List, Optional, Tuple

DOMAINS = ("web", "code", "wiki", "books", "science", "math", "conversation", "other")


@dataclass
class DataMixConfig:
    weights: Dict[str, float] = field(default_factory=lambda: {
        "web": 0.35, "code": 0.20, "wiki": 0.12, "books": 0.10, "science": 0.08, "math": 0.07,
        "conversation": 0.05, "other": 0.03})
    min_doc_length: int = 50
    max_doc_length: int = 100_000
    min_quality_score: float = 0.3
    dedup_threshold: float = 0.8
    target_total_tokens: int = 2_000_000_000_000
    shuffle_seed: int = 42

    @classmethod
    def from_yaml(cls, path: str) -> "DataMixConfig":
        import yaml
        d = yaml.safe_load(open(path)) or {}
        known = {k: v for k, v in d.items() if k in cls.__dataclass_fields__}
        return cls(**known)


class DomainClassifier:
    MARKERS: Dict[str, List[str]] = {
        "code": [r"\bdef \w+\(", r"\bclass \w+[:(]", r"#include\s*<", r"\breturn\b", r"[{};]\s*$", r"```",
                 r"\bimport \w+", r"\bfunction\s*\w*\(", r"=>", r"\bpublic\b|\bprivate\b"],
        "math": [r"\\frac|\\sum|\\int|\\sqrt", r"\$[^$]+\$", r"\btheorem\b|\blemma\b|\bproof\b", r"[=<>]\s*-?\d",
                 r"\b(sin|cos|log|lim)\b"],
        "wiki": [r"\[\[[^\]]+\]\]", r"\{\{[^}]+\}\}", r"^==+ .* ==+$", r"<ref", r"Category:"],
        "books": [r"\bchapter\s+[ivxlc\d]+\b", r"[\"“][^\"”]{15,}[\"”]", r"\b(said|asked|replied)\b"],
        "science": [r"\bet al\.", r"\bdoi:", r"\b(fig\.|figure)\s*\d", r"\bp\s*[<>]\s*0?\.\d", r"\bhypothes[ie]s\b",
                    r"\b(abstract|methods|results)\b"],
        "conversation": [r"^(user|assistant|human|ai|q|a):", r"\?\s*$"],
        "web": [r"https?://", r"\b(click|subscribe|cookie|login|home page)\b", r"©|\ball rights reserved\b"],
    }

    def __init__(self):
        self._re = {d: [re.compile(p, re.IGNORECASE | re.MULTILINE) for p in ps] for d, ps in self.MARKERS.items()}

    def classify(self, text: str) -> Tuple[str, float, Dict[str, float]]:
        n = max(1, len(text) / 1000.0)
        scores = {d: sum(len(r.findall(text)) for r in rs) / n for d, rs in self._re.items()}
        best = max(scores, key=scores.get)
        tot = sum(scores.values())
        if tot == 0:
            return "other", 0.0, scores
        return best, scores[best] / tot, scores


class QualityScorer:
    def __init__(self, min_length: int = 50, max_length: int = 100_000, optimal_length: int = 2000):
        self.min_length, self.max_length, self.optimal_length = min_length, max_length, optimal_length

    def score(self, text: str) -> Tuple[float, Dict[str, float]]:
        if not text or len(text) < self.min_length:
            return 0.0, {"length": 0.0}
        words = text.split()
        parts = {"length": self._length(len(text)), "repetition": self._repetition(words),
                 "diversity": self._diversity(words), "structure": self._structure(text)}
        w = {"length": 0.2, "repetition": 0.35, "diversity": 0.3, "structure": 0.15}
        return sum(parts[k] * w[k] for k in parts), parts

    def _length(self, L: int) -> float:
        if L > self.max_length:
            return 0.2
        x = math.log(L / self.optimal_length)
        return math.exp(-x * x)

    @staticmethod
    def _repetition(words: List[str]) -> float:
        if len(words) < 20:
            return 0.5
        grams = [" ".join(words[i:i + 3]).lower() for i in range(len(words) - 2)]
        dup = len(grams) - len(set(grams))
        return max(0.0, 1.0 - 4.0 * dup / max(1, len(grams)))

    @staticmethod
    def _diversity(words: List[str]) -> float:
        if len(words) < 30:
            return 0.3
        ttr = len(set(w.lower() for w in words)) / len(words)
        return min(1.0, ttr / max(0.1, 0.6 - 1e-4 * len(words)))

    @staticmethod
    def _structure(text: str) -> float:
        s = 0.5
        paras = [p for p in text.split("\n\n") if p.strip()]
        s += 0.15 * (len(paras) >= 2) + 0.1 * (len(paras) >= 5)
        s += min(0.15, 0.02 * len(set(re.findall(r"[.,!?;:'\"-]", text))))
        upper = sum(c.isupper() for c in text) / max(1, len(text))
        s -= 0.2 * (upper > 0.3) + 0.15 * (text.count("\n") / max(1, len(text)) > 0.05)
        return max(0.0, min(1.0, s))


class Deduplicator:
    """Exact (content hash) and near (MinHash-LSH) duplicate detection over a stream."""

    _P = (1 << 61) - 1

    def __init__(self, threshold: float = 0.8, num_hashes: int = 128, num_bands: int = 16, shingle: int = 5):
        self.threshold, self.k, self.bands, self.shingle = threshold, num_hashes, num_bands, shingle
        self.rows = num_hashes // num_bands
        rng = random.Random(1234)
        self.ab = [(rng.randrange(1, self._P), rng.randrange(0, self._P)) for _ in range(num_hashes)]
        self.exact = set()
        self.buckets: List[Dict[tuple, List[int]]] = [defaultdict(list) for _ in range(num_bands)]
        self.sigs: List[List[int]] = []
        self.stats = Counter()

    def signature(self, text: str) -> List[int]:
        toks = text.lower().split()
        sh = {" ".join(toks[i:i + self.shingle]) for i in range(max(1, len(toks) - self.shingle + 1))}
        hs = [int.from_bytes(hashlib.blake2b(s.encode(), digest_size=8).digest(), "little") for s in sh]
        return [min((a * h + b) % self._P for h in hs) for a, b in self.ab]

    @staticmethod
    def similarity(s1: List[int], s2: List[int]) -> float:
        return sum(x == y for x, y in zip(s1, s2)) / len(s1)

    def is_duplicate(self, text: str) -> Tuple[bool, str]:
        h = hashlib.sha1(text.strip().encode()).hexdigest()
        if h in self.exact:
            self.stats["exact"] += 1
            return True, "exact"
        self.exact.add(h)
        sig = self.signature(text)
        cands = set()
        for b in range(self.bands):
            cands.update(self.buckets[b].get(tuple(sig[b * self.rows:(b + 1) * self.rows]), ()))
        for c in cands:
            if self.similarity(sig, self.sigs[c]) >= self.threshold:
                self.stats["near"] += 1
                return True, "near"
        idx = len(self.sigs)
        self.sigs.append(sig)
        for b in range(self.bands):
            self.buckets[b][tuple(sig[b * self.rows:(b + 1) * self.rows])].append(idx)
        self.stats["unique"] += 1
        return False, ""

    def get_stats(self) -> dict:
        return dict(self.stats)


class ContentFilter:
    PATTERNS = [(r"(?i)lorem ipsum", "placeholder text"), (r"(.)\1{30,}", "character run"),
                (r"(?i)\b(viagra|casino bonus|click here to win)\b", "spam"),
                (r"[\x00-\x08\x0e-\x1f]", "control characters")]

    def __init__(self):
        self._re = [(re.compile(p), why) for p, why in self.PATTERNS]
        self.stats = Counter()

    def should_filter(self, text: str) -> Tuple[bool, str]:
        for r, why in self._re:
            if r.search(text):
                self.stats[why] += 1
                return True, why
        return False, ""

    def get_stats(self) -> dict:
        return dict(self.stats)


class DataMixer:
    def __init__(self, config: DataMixConfig):
        self.config = config
        self.pools: Dict[str, List[Tuple[str, float]]] = defaultdict(list)
        self.rng = random.Random(config.shuffle_seed)

    def add_document(self, text: str, domain: str, quality: float) -> None:
        self.pools[domain if domain in self.config.weights else "other"].append((text, quality))

    def sample_batch(self, batch_size: int) -> List[str]:
        doms = [d for d in self.config.weights if self.pools.get(d)]
        if not doms:
            return []
        w = [self.config.weights[d] for d in doms]
        return [self.rng.choice(self.pools[d])[0] for d in self.rng.choices(doms, weights=w, k=batch_size)]

    def get_distribution(self) -> Dict[str, int]:
        return {d: len(p) for d, p in self.pools.items()}

    def get_all_documents(self, shuffle: bool = True) -> Iterator[Tuple[str, str]]:
        docs = [(t, d) for d, p in self.pools.items() for t, _ in p]
        if shuffle:
            self.rng.shuffle(docs)
        yield from docs


class MultiFormatReader:
    CODE_EXT = {".py", ".js", ".ts", ".c", ".cc", ".cpp", ".h", ".hpp", ".cu", ".java", ".go", ".rs", ".rb", ".sh"}

    def __init__(self, extract_pdf: bool = False):
        self.extract_pdf = extract_pdf
        self.stats = Counter()

    def read_file(self, path: str) -> Iterator[Tuple[str, str]]:
        """Yield (text, domain hint or '') for each document of a file."""
        ext = os.path.splitext(path)[1].lower()
        try:
            if ext in (".jsonl", ".json"):
                yield from self._json(path, ext)
            elif ext in (".csv", ".tsv"):
                with open(path, newline="", encoding="utf-8", errors="replace") as f:
                    for row in csv.DictReader(f, delimiter="\t" if ext == ".tsv" else ","):
                        t = row.get("text") or " ".join(v for v in row.values() if v)
                        if t:
                            yield t, ""
            elif ext in (".html", ".htm", ".xml"):
                raw = open(path, encoding="utf-8", errors="replace").read()
                yield html.unescape(re.sub(r"<[^>]+>", " ", re.sub(r"(?is)<(script|style).*?</\1>", " ", raw))), "web"
            elif ext in (".md", ".markdown"):
                raw = open(path, encoding="utf-8", errors="replace").read()
                yield re.sub(r"!\[[^\]]*\]\([^)]*\)|\[([^\]]*)\]\([^)]*\)", r"\1", raw), ""
            elif ext == ".tex":
                yield open(path, encoding="utf-8", errors="replace").read(), "math"
            elif ext in self.CODE_EXT:
                yield open(path, encoding="utf-8", errors="replace").read(), "code"
            else:
                raw = open(path, encoding="utf-8", errors="replace").read()
                for doc in raw.split("\n\n\n"):
                    if doc.strip():
                        yield doc, ""
            self.stats[ext or "none"] += 1
        except (OSError, UnicodeError, json.JSONDecodeError) as e:
            self.stats["errors"] += 1

    def _json(self, path, ext):
        with open(path, encoding="utf-8", errors="replace") as f:
            objs = (json.loads(l) for l in f if l.strip()) if ext == ".jsonl" else iter(json.load(f) or [])
            for o in objs:
                if isinstance(o, str):
                    yield o, ""
                elif isinstance(o, dict):
                    t = o.get("text") or o.get("content") or " ".join(str(o[k]) for k in ("question", "answer")
                                                                      if k in o)
                    if t:
                        yield t, o.get("domain", "")

    def get_stats(self) -> dict:
        return dict(self.stats)


class DataPipeline:
    def __init__(self, config: Optional[DataMixConfig] = None, override_domain: Optional[str] = None):
        self.config = config or DataMixConfig()
        self.override_domain = override_domain
        self.reader = MultiFormatReader()
        self.classifier = DomainClassifier()
        self.scorer = QualityScorer(self.config.min_doc_length, self.config.max_doc_length)
        self.dedup = Deduplicator(self.config.dedup_threshold)
        self.filter = ContentFilter()
        self.mixer = DataMixer(self.config)
        self.stats = Counter()

    def process_text(self, text: str, hint: str = "") -> Optional[str]:
        self.stats["seen"] += 1
        if not (self.config.min_doc_length <= len(text) <= self.config.max_doc_length):
            self.stats["length_rejected"] += 1
            return None
        if self.filter.should_filter(text)[0]:
            self.stats["filtered"] += 1
            return None
        q, _ = self.scorer.score(text)
        if q < self.config.min_quality_score:
            self.stats["low_quality"] += 1
            return None
        if self.dedup.is_duplicate(text)[0]:
            self.stats["duplicates"] += 1
            return None
        dom = self.override_domain or hint or self.classifier.classify(text)[0]
        self.mixer.add_document(text, dom, q)
        self.stats["kept"] += 1
        return dom

    def process_file(self, path: str) -> dict:
        kept = Counter()
        for text, hint in self.reader.read_file(path):
            d = self.process_text(text, hint)
            if d:
                kept[d] += 1
        return dict(kept)

    def process_directory(self, input_dir: str) -> dict:
        out = Counter()
        for root, _, files in os.walk(input_dir):
            for f in sorted(files):
                out.update(self.process_file(os.path.join(root, f)))
        return dict(out)

    def generate_report(self) -> str:
        lines = ["data pipeline report", f"  documents seen {self.stats['seen']}, kept {self.stats['kept']}"]
        for k in ("length_rejected", "filtered", "low_quality", "duplicates"):
            lines.append(f"  {k:16s} {self.stats[k]}")
        dist = self.mixer.get_distribution()
        tot = max(1, sum(dist.values()))
        for d in DOMAINS:
            lines.append(f"  {d:13s} {dist.get(d, 0):8d} ({100 * dist.get(d, 0) / tot:5.1f}%, "
                         f"target {100 * self.config.weights.get(d, 0):.0f}%)")
        return "\n".join(lines)

    def save_mixer_state(self, output_dir: str) -> None:
        os.makedirs(output_dir, exist_ok=True)
        with open(os.path.join(output_dir, "mixed.jsonl"), "w", encoding="utf-8") as f:
            for text, dom in self.mixer.get_all_documents():
                f.write(json.dumps({"text": text, "domain": dom}, ensure_ascii=False) + "\n")
        with open(os.path.join(output_dir, "pipeline_stats.json"), "w") as f:
            json.dump({"stats": dict(self.stats), "distribution": self.mixer.get_distribution(),
                       "dedup": self.dedup.get_stats(), "filter": self.filter.get_stats(),
                       "reader": self.reader.get_stats()}, f, indent=2)
