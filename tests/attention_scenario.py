"""The scenarios of the reference's own attention tests
(tests/test_sliding_attention_degree_parity.mojo and
tests/test_full_attention_degree_parity.mojo, at degree 1), restated for this
library's tests: three sequences on 64-row pages (a two-page ring for the
sliding layer, 3 or 5 pages for the full layer), ten steps of prefill chunks
and decode tokens, hashed token content (content_value), unit q/k gains and
an identity rotary table, and the tests' float reference (reference_head:
exact exp, f32 running sums) with their acceptance bound, 0.05 absolute per
output element.  Line numbers below are the sliding test's unless marked."""
import numpy as np

# sliding layer (the sliding test, :15-32)
HEAD_DIM, NUM_Q, NUM_KV = 256, 16, 8
GQA = NUM_Q // NUM_KV
PAGE_LEN, WINDOW, RING_PAGES = 64, 64, 2
NUM_PAGES = 6
ROPE_ROWS = 512
TOL = 0.05
# full layer (the full test, :15-31 and :43-59 sequence_pages)
FULL_HEAD_DIM, FULL_NUM_Q, FULL_NUM_KV = 512, 16, 2
FULL_NUM_PAGES = 12
FULL_SEQ_PAGES = {0: (3, 7, 11), 1: (0, 5, 9), 2: (2, 4, 6, 8, 10)}

# (sequence, first position, token count) runs of each step (:370-413)
STEPS = [
    [(0, 0, 64)],
    [(0, 64, 64)],
    [(0, 128, 22), (1, 0, 42)],
    [(1, 42, 64)],
    [(1, 106, 14), (2, 0, 50)],
    [(2, 50, 64)],
    [(2, 114, 64)],
    [(0, 150, 1), (1, 120, 1), (2, 178, 22)],
    [(0, 151, 1), (1, 121, 1), (2, 200, 1)],
    [(0, 152, 1)],
]
SEQ_PAGES = {0: (3, 1), 1: (0, 4), 2: (2, 5)}   # :44-53 sequence_pages


def content_value(key, column, salt):
    """:56-63 content_value, vectorised over `column` (uint64 wrap-around)."""
    c = np.asarray(column, dtype=np.uint64)
    with np.errstate(over="ignore"):
        h = (np.uint64(key) * np.uint64(2654435761) + c * np.uint64(2246822519)
             + np.uint64(salt) * np.uint64(3266489917))
        h ^= h >> np.uint64(13)
        h = h * np.uint64(1099511628211)
        h ^= h >> np.uint64(29)
    return (np.asarray(h % np.uint64(17), np.int64) - 8).astype(np.float32) * np.float32(0.05)


def to_bf16(a):
    b = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((b + ((b >> 16) & 1) + 0x7FFF) >> 16).astype(np.uint16)


def step_tokens(step):
    """(sequence, position) of every token of a step, and its runs as
    (buf_start, base_pos, sequence)."""
    toks, runs = [], []
    for seq, start, count in STEPS[step]:
        runs.append((len(toks), start, seq))
        toks += [(seq, p) for p in range(start, start + count)]
    return toks, runs


def step_inputs(step, head_dim=HEAD_DIM, num_q=NUM_Q, num_kv=NUM_KV):
    """bf16 q [T][num_q*head_dim], k, v [T][num_kv*head_dim] of a step
    (sliding test :171-183, full test :131-141)."""
    toks, _ = step_tokens(step)
    T = len(toks)
    q = np.empty((T, num_q * head_dim), np.uint16)
    k = np.empty((T, num_kv * head_dim), np.uint16)
    v = np.empty_like(k)
    for t, (seq, pos) in enumerate(toks):
        key = seq * 512 + pos
        q[t] = to_bf16(content_value(key, np.arange(num_q * head_dim), 1))
        k[t] = to_bf16(content_value(key, np.arange(num_kv * head_dim), 2))
        v[t] = to_bf16(content_value(key, np.arange(num_kv * head_dim), 3))
    return q, k, v


def ring_slot(pos, seq):
    """:89-90 ring_slot."""
    pages = SEQ_PAGES[seq]
    return pages[(pos // PAGE_LEN) % RING_PAGES] * PAGE_LEN + pos % PAGE_LEN


def base_rows(seq):
    return np.array([p * PAGE_LEN for p in SEQ_PAGES[seq]], np.int32)


def window_slots(seq, pos):
    lo = max(0, pos - WINDOW + 1)
    return [ring_slot(p, seq) for p in range(lo, pos + 1)]


def full_slot(pos, seq):
    """The full test's slot of a position at degree 1 (:301-302)."""
    pages = FULL_SEQ_PAGES[seq]
    return pages[pos // PAGE_LEN] * PAGE_LEN + pos % PAGE_LEN


def full_base_rows(seq):
    return np.array([p * PAGE_LEN for p in FULL_SEQ_PAGES[seq]], np.int32)


def full_slots(seq, pos):
    return [full_slot(p, seq) for p in range(pos + 1)]


def reference_head(kc, ks, vc, vs, seq, pos, q_row, qf, head, full=False):
    """reference_head of the sliding test (:93-138) or, with full, of the full
    test at degree 1 (:276-329): f32 online softmax with exact exp."""
    hd = FULL_HEAD_DIM if full else HEAD_DIM
    kvh = head // ((FULL_NUM_Q // FULL_NUM_KV) if full else GQA)
    inv127 = np.float32(1.0) / np.float32(127.0)
    inv127sq = np.float32(inv127 * inv127)
    m, l = np.float32(-1e30), np.float32(0.0)
    acc = np.zeros(hd, np.float32)
    q = q_row.astype(np.int64)
    for slot in (full_slots(seq, pos) if full else window_slots(seq, pos)):
        kr = kc[slot, kvh * hd:(kvh + 1) * hd].astype(np.int64)
        dot = np.float32(int((kr * q).sum()))
        s = np.float32(np.float32(np.float32(dot * qf) * ks[slot, kvh]) * inv127sq)
        m_new = s if s > m else m
        corr = np.float32(np.exp(np.float32(m - m_new)))
        w = np.float32(np.exp(np.float32(s - m_new)))
        l = np.float32(l * corr + w)
        vw = np.float32(np.float32(w * vs[slot, kvh]) * inv127)
        vr = vc[slot, kvh * hd:(kvh + 1) * hd].astype(np.float32)
        acc = acc * corr + vr * vw
        m = m_new
    if l > 0:
        acc = acc * (np.float32(1.0) / l)
    return acc


def identity_rope(rope_half=HEAD_DIM // 2):
    return np.ones((ROPE_ROWS, rope_half), np.float32), np.zeros((ROPE_ROWS, rope_half), np.float32)


def unit_gain(head_dim=HEAD_DIM):
    return to_bf16(np.ones(head_dim, np.float32))
