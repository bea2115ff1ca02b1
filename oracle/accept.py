"""CPU restatement of WPT's speculative-decoding acceptance step, in numpy.

TEST INFRASTRUCTURE ONLY (the checker): only `tests/`, `__graft_entry__.smoke()`
and the CPU legs of `bench.py` may import it.

Follows packages/wpt-inference/src/wpt_inference/__init__.py:
    probabilities  :173-179  scores / temperature, top-k mask (ties kept:
                             `scores < v[..., [-1]]`), softmax, all float32
    accept loop    :210-222  keep draft j iff u_j * q[j, tok] < p[j, tok];
                             on the first rejection draw from
                             normalize(max(0, p[j] - q[j])) and stop; when
                             every draft is kept draw one more from p[n]

The reference draws with torch.rand (one scalar per draft) and
torch.multinomial. This restatement takes the draws as explicit inputs so
that the GPU kernel can be checked bit for bit: uniforms[i, j] is draft j's
acceptance draw, resample[i] the single draw of the row's last token, turned
into a token by inverse CDF: the first vocabulary index whose float64
running sum of the (float32) weights exceeds resample[i] times their total.
tests/golden/make_golden.py pins this against the reference's own
Writer._speculate with torch.rand and torch.multinomial replaced by those
two rules.
"""

import numpy as np


def head_scores(h, weight, round_bf16=True):
    """model.py:267,471: the output head, h (R, D) @ weight (V, D)^T (an
    nn.Linear without bias), in float64 here; round_bf16 rounds each score to
    bf16 (round to nearest even), as the reference's head under bf16 autocast
    returns it before .float()."""
    s = np.asarray(h, np.float64) @ np.asarray(weight, np.float64).T
    if not round_bf16:
        return s.astype(np.float32)
    bits = s.astype(np.float32).view(np.uint32).astype(np.uint64)
    bits = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16 << 16
    return bits.astype(np.uint32).view(np.float32)


def probabilities(scores, temperature, top_k):
    """__init__.py:173-179 in float32: (..., V) -> (..., V)."""
    x = np.asarray(scores, np.float32) / np.float32(temperature)
    if top_k is not None:
        kk = min(int(top_k), x.shape[-1])
        kth = -np.partition(-x, kk - 1, axis=-1)[..., kk - 1:kk]
        x = np.where(x < kth, np.float32(-np.inf), x)
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp(x - m, dtype=np.float32)
    return (e / np.sum(e, axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def inverse_cdf(weights, u):
    """The first index whose float64 running sum of weights exceeds u * total."""
    cs = np.cumsum(np.asarray(weights, np.float64))
    target = float(u) * cs[-1]
    return int(min(np.searchsorted(cs, target, side="right"), len(cs) - 1))


def accept(scores, drafted, q, uniforms, resample, temperature=1.0, top_k=None, lengths=None):
    """scores (R, n + 1, V) the target model's logits at each draft's place
    and one after; drafted (R, n) the draft tokens; q (R, n, V) the
    drafter's probabilities; uniforms (R, n); resample (R,); lengths (R,)
    drafts verified per row (default n).

    Returns (tokens (R, n + 1) int64, -1 padded; accepted (R,) int64): each
    row's kept drafts then its one drawn token, and how many drafts it kept.
    """
    scores = np.asarray(scores, np.float32)
    q = np.asarray(q, np.float32)
    drafted = np.asarray(drafted, np.int64)
    uniforms = np.asarray(uniforms, np.float32)
    resample = np.asarray(resample, np.float32)
    R, n1, V = scores.shape
    n = n1 - 1
    lengths = np.full(R, n, np.int64) if lengths is None else np.asarray(lengths, np.int64)
    tokens = np.full((R, n + 1), -1, np.int64)
    accepted = np.zeros(R, np.int64)
    for i in range(R):
        ni = int(lengths[i])
        p = probabilities(scores[i, :ni + 1], temperature, top_k)
        kept = []
        rejected = False
        for j in range(ni):
            tok = int(drafted[i, j])
            if np.float32(uniforms[i, j]) * q[i, j, tok] < p[j, tok]:
                kept.append(tok)
                continue
            rest = np.maximum(p[j] - q[i, j], np.float32(0))
            kept.append(inverse_cdf(rest, resample[i]))
            rejected = True
            break
        if not rejected:
            kept.append(inverse_cdf(p[ni], resample[i]))
        accepted[i] = len(kept) - 1
        tokens[i, :len(kept)] = kept
    return tokens, accepted
