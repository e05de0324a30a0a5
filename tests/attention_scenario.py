"""The scenario of the reference's own sliding-attention test
(tests/test_sliding_attention_degree_parity.mojo), restated for this
library's tests: three sequences on two-page rings of 64-row pages, ten steps
of prefill chunks and decode tokens, hashed token content (:56-63
content_value), unit q/k gains and an identity rotary table (:340-346), and
its float reference (:93-138 reference_head: exact exp, f32 running sums)
with its acceptance bound, 0.05 absolute per output element (:243)."""
import numpy as np

HEAD_DIM, NUM_Q, NUM_KV = 256, 16, 8
GQA = NUM_Q // NUM_KV
PAGE_LEN, WINDOW, RING_PAGES = 64, 64, 2
NUM_PAGES = 6
ROPE_ROWS = 512
TOL = 0.05

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
M64 = (1 << 64) - 1


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


def step_inputs(step):
    """bf16 q [T][16*256], k, v [T][8*256] of a step (:171-183)."""
    toks, _ = step_tokens(step)
    T = len(toks)
    q = np.empty((T, NUM_Q * HEAD_DIM), np.uint16)
    k = np.empty((T, NUM_KV * HEAD_DIM), np.uint16)
    v = np.empty_like(k)
    for t, (seq, pos) in enumerate(toks):
        key = seq * 512 + pos
        q[t] = to_bf16(content_value(key, np.arange(NUM_Q * HEAD_DIM), 1))
        k[t] = to_bf16(content_value(key, np.arange(NUM_KV * HEAD_DIM), 2))
        v[t] = to_bf16(content_value(key, np.arange(NUM_KV * HEAD_DIM), 3))
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


def reference_head(kc, ks, vc, vs, seq, pos, q_row, qf, head):
    """:93-138 reference_head: f32 online softmax with exact exp."""
    kvh = head // GQA
    inv127 = np.float32(1.0) / np.float32(127.0)
    inv127sq = np.float32(inv127 * inv127)
    m, l = np.float32(-1e30), np.float32(0.0)
    acc = np.zeros(HEAD_DIM, np.float32)
    q = q_row.astype(np.int64)
    for slot in window_slots(seq, pos):
        kr = kc[slot, kvh * HEAD_DIM:(kvh + 1) * HEAD_DIM].astype(np.int64)
        dot = np.float32(int((kr * q).sum()))
        s = np.float32(np.float32(np.float32(dot * qf) * ks[slot, kvh]) * inv127sq)
        m_new = s if s > m else m
        corr = np.float32(np.exp(np.float32(m - m_new)))
        w = np.float32(np.exp(np.float32(s - m_new)))
        l = np.float32(l * corr + w)
        vw = np.float32(np.float32(w * vs[slot, kvh]) * inv127)
        vr = vc[slot, kvh * HEAD_DIM:(kvh + 1) * HEAD_DIM].astype(np.float32)
        acc = acc * corr + vr * vw
        m = m_new
    if l > 0:
        acc = acc * (np.float32(1.0) / l)
    return acc


def identity_rope():
    half = HEAD_DIM // 2
    return np.ones((ROPE_ROWS, half), np.float32), np.zeros((ROPE_ROWS, half), np.float32)


def unit_gain():
    return to_bf16(np.ones(HEAD_DIM, np.float32))
