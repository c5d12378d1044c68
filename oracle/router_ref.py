"""TEST INFRASTRUCTURE ONLY: plain-Python restatement of the reference's request
encoding (below the tokenizer) and hierarchical router, the checker for
libj1's j1_encode_sequence / j1_engine_logits_tokenized / j1_router_route_many.

Follows, step by step:
  * Encoder::sequence        src/encode.rs:138-195 (OPTION_TOKENS = 48, encode.rs:12)
  * Request::validate        src/request.rs:132-146
  * display_probabilities    src/request.rs:150-161
  * argmax                   src/request.rs:164-172
  * Router::new / validate / key / score / confident_winner / route_many
                             src/router.rs:39-210
The text-level parts (tokenizing, replacing the mask token's text) are the
caller's: requests here carry token ids, as in the C ABI.
"""
import math
from collections import OrderedDict
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence

OPTION_TOKENS = 48


class RefError(ValueError):
    pass


@dataclass
class Req:
    head: List[int]
    options: List[List[int]]
    state: List[int]
    qtype: int = 0  # 0 choice, 1 score, 2 noul


@dataclass
class EncOpts:
    cls_id: int
    sep_id: int
    mask_id: int
    max_length: int = 512
    head_length: int = 256
    strict: bool = False


def encode_sequence(o: EncOpts, r: Req):
    """Encoder::sequence on ids -> (ids, markers, truncated) (encode.rs:138-195)."""
    if o.head_length + 4 >= o.max_length:  # Encoder::from_parts (encode.rs:66-68)
        raise RefError("max_length must leave room beyond the question head")
    if not r.options:
        raise RefError("request has no options")
    if any(o.mask_id in t for t in [r.head, r.state] + list(r.options)):
        raise RefError("Reserved model marker in request" if o.strict else "mask token id inside request tokens")
    if o.strict and any(len(x) > OPTION_TOKENS for x in r.options):
        raise RefError("Option exceeds 48-token model contract")
    options = [[o.mask_id] + list(x[:OPTION_TOKENS]) for x in r.options]
    budget = o.head_length - sum(len(v) for v in options)
    if budget < 16:
        per_option = max((o.head_length - 16) // len(options), 4)  # div_euclid == floor for n > 0
        options = [v[:per_option] for v in options]
        budget = o.head_length - sum(len(v) for v in options)
    if o.strict and (len(r.head) > budget or any(len(v) != len(x) + 1 for v, x in zip(options, r.options))):
        raise RefError("Question/options exceed lossless head budget")
    ids = [o.cls_id] + list(r.head[:min(len(r.head), max(budget, 8))]) + [o.sep_id]
    markers = []
    for v in options:
        markers.append(len(ids))
        ids.extend(v)
    ids.append(o.sep_id)
    room = o.max_length - len(ids) - 1
    if room < 1:
        raise RefError("Question/options exceed sequence budget; shorten descriptions")
    if o.strict and len(r.state) > room:
        raise RefError("Game state exceeds lossless context budget")
    ids.extend(r.state[:room])
    ids.append(o.sep_id)
    return ids, markers, len(r.state) > room


def validate_request(r: Req):
    """Request::validate (request.rs:132-146) on what survives tokenization."""
    if not (2 <= len(r.options) <= 20) or any(len(x) == 0 for x in r.options):
        raise RefError("options must contain 2–20 nonempty rendered descriptions")
    if r.qtype == 2 and len(r.options) != 2:
        raise RefError("noul options must be ordered [false, true]")


def argmax(values) -> int:
    best = 0
    for i, v in enumerate(values):
        if v > values[best]:
            best = i
    return best


def display_probabilities(values: Sequence[float]) -> List[float]:
    if not values:
        return []
    w = argmax(values)
    if values[w] > 0.95 and all(i == w or v < 0.045 for i, v in enumerate(values)):
        return [1.0 if i == w else 0.0 for i in range(len(values))]
    visible = [v if v >= 0.01 else 0.0 for v in values]
    total = sum(visible)
    return [v / total for v in visible]


def confident_winner(scores: Sequence[float], best: int) -> bool:
    s = [float(x) for x in scores]
    runner_up = -math.inf
    for i, v in enumerate(s):
        if i != best:
            runner_up = max(runner_up, v)
    if runner_up - s[best] >= math.log(0.045 / 0.95):
        return False
    total = sum(math.exp(v - s[best]) for v in s)
    return 1.0 / total > 0.95 and math.exp(runner_up - s[best]) / total < 0.045


def f32(x) -> float:
    """Round a Python float to float32 (the logits are f32 in the reference)."""
    import struct
    return struct.unpack("f", struct.pack("f", x))[0]


@dataclass
class RouteResult:
    index: int
    candidates: List[int]
    probabilities: List[float]
    rounds: int
    hierarchical: bool


class Router:
    """Router (router.rs). `logits(rows)` scores a list of Req and returns per-row f32 logits."""

    def __init__(self, logits: Callable[[List[Req]], List[List[float]]], width=20, survivors=2, batch_size=16,
                 cache_size=0, max_options=4096):
        if not (2 <= width <= 20) or not (1 <= survivors < width):
            raise RefError("Require 2 <= width <= 20 and 1 <= survivors < width")
        if batch_size < 1 or max_options < width:
            raise RefError("Invalid batch/cache/capacity limit")
        self.logits, self.width, self.survivors = logits, width, survivors
        self.batch_size, self.max_options = batch_size, max_options
        self.cache: Optional[OrderedDict] = OrderedDict() if cache_size > 0 else None
        self.cache_size = cache_size

    def clear_cache(self):
        if self.cache is not None:
            self.cache.clear()

    def _validate(self, r: Req):
        if not (2 <= len(r.options) <= self.max_options):
            raise RefError("Expected 2–%d options" % self.max_options)
        if any(len(x) == 0 for x in r.options):
            raise RefError("Options must be nonempty strings")
        if r.qtype == 2 and len(r.options) != 2:
            raise RefError("noul requires [false, true]")
        if r.qtype != 0 and len(r.options) > self.width:
            raise RefError("Hierarchical routing supports choice decisions only")

    @staticmethod
    def _key(r: Req):
        return (r.qtype, tuple(r.head), tuple(r.state), tuple(tuple(x) for x in r.options))

    def _score(self, jobs: List[Req]):
        values: List[Optional[List[float]]] = [None] * len(jobs)
        missing, index, hits = [], {}, 0
        for i, row in enumerate(jobs):
            key = self._key(row)
            if self.cache is not None and key in self.cache:
                self.cache.move_to_end(key)  # LruCache::get promotes
                values[i] = list(self.cache[key])
                hits += 1
                continue
            if key in index:
                missing[index[key]][1].append(i)
                hits += 1
            else:
                index[key] = len(missing)
                missing.append((key, [i]))
        for c0 in range(0, len(missing), self.batch_size):
            chunk = missing[c0:c0 + self.batch_size]
            output = self.logits([jobs[idx[0]] for _, idx in chunk])
            if len(output) != len(chunk):
                raise RefError("Engine returned the wrong number of rows")
            for (key, indices), scores in zip(chunk, output):
                scores = [f32(v) for v in scores]
                if len(scores) != len(jobs[indices[0]].options) or any(not math.isfinite(v) for v in scores):
                    raise RefError("Engine logits must be finite and match option count")
                for i in indices:
                    values[i] = scores
                if self.cache is not None:
                    if key in self.cache:
                        self.cache.move_to_end(key)
                    elif len(self.cache) >= self.cache_size:
                        self.cache.popitem(last=False)
                    self.cache[key] = scores
        return values, len(missing), hits

    def route_many(self, rows: List[Req]):
        for r in rows:
            self._validate(r)
        candidates = [list(range(len(r.options))) for r in rows]
        results: List[Optional[RouteResult]] = [None] * len(rows)
        rounds = [0] * len(rows)
        model_rows = hits = 0
        while any(x is None for x in results):
            jobs, layout = [], []
            for i, row in enumerate(rows):
                if results[i] is not None:
                    continue
                rounds[i] += 1
                current, candidates[i] = candidates[i], []
                last = len(current) <= self.width
                for g0 in range(0, len(current), self.width):
                    group = current[g0:g0 + self.width]
                    if len(group) == 1:
                        candidates[i].extend(group)
                        continue
                    jobs.append(Req(row.head, [row.options[k] for k in group], row.state, row.qtype))
                    layout.append((i, group, last))
            scored, used, cached = self._score(jobs)
            model_rows += used
            hits += cached
            for (i, group, last), scores in zip(layout, scored):
                best = argmax(scores)
                if last:
                    mx = max(scores)
                    weights = [math.exp(x - mx) for x in scores]
                    total = sum(weights)
                    hier = len(rows[i].options) > self.width
                    results[i] = RouteResult(group[best], list(group),
                                             display_probabilities([w / total for w in weights]), rounds[i], hier)
                elif confident_winner(scores, best):
                    candidates[i].append(group[best])
                else:
                    remaining = list(range(len(group)))
                    chosen = []
                    for _ in range(min(self.survivors, len(group))):
                        local = [scores[k] for k in remaining]
                        chosen.append(group[remaining.pop(argmax(local))])
                    chosen.sort()
                    candidates[i].extend(chosen)
        return results, model_rows, hits


QNAMES = {0: "choice", 1: "score", 2: "noul"}


def encode_text(tokenize, mask_token: str, o: EncOpts, state: str, question: str, options, qtype: int = 0):
    """Encoder::sequence with its text part (encode.rs:138-150): strict refusal of the mask
    token's text, mask text replaced by a space, the head / option / state text forms,
    tokenized by `tokenize` (the checkpoint tokenizer), then the layout on ids."""
    if o.strict and any(mask_token in t for t in [state, question] + list(options)):
        raise RefError("Reserved model marker in request")

    def clean(t):
        return t.replace(mask_token, " ")

    head = tokenize("%s question: %s" % (QNAMES[qtype], clean(question)))
    opts = [tokenize(" " + clean(x)) for x in options]
    state_ids = tokenize(clean(state))
    return encode_sequence(o, Req(list(head), [list(x) for x in opts], list(state_ids), qtype))
