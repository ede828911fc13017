"""Streaming text of sessions decoded together (lfm_text_*, host code, no GPU)
against the Python restatement of the reference's Utf8Stream / StreamDecoder
(tokenizer/src/stream.rs) and DecodedText (engine/src/text_output.rs).

Pins: the known-answer cases of the reference's streaming tests
(tokenizer/tests/streaming.rs:99-141, both invalid-byte policies and the end of
stream), and the property of engine/tests/text_stream.rs: text streamed
chunk by chunk through the cleanup equals the whole-sequence cleanup, on the
same kind of xorshift-generated samples (spaces, apostrophes, punctuation,
multi-byte characters), split at arbitrary byte boundaries.
"""

import numpy as np
import pytest

import text_stream as ref

BYTES = [bytes([b]) for b in range(256)]  # one token per byte value


def streams(pieces, n=1, clean=False, replace=False):
    import lfm2_b200
    return lfm2_b200.TextStreams(pieces, n, clean_spaces=clean, replace_invalid=replace)


def push_bytes(t, data, session=0):
    out = t.push([session] * len(data), list(data))
    return b"".join(out)


def test_invalid_bytes_replace_policy():
    t = streams(BYTES + [b"ok"], replace=True)
    rep = "�".encode()
    assert push_bytes(t, b"a\xffb") == b"a" + rep + b"b"
    assert push_bytes(t, b"\xf0\x9f") == b""
    assert push_bytes(t, b"x") == rep + b"x"
    assert push_bytes(t, b"\xed\xa0\x80") == rep * 3  # surrogate encoding is invalid
    assert push_bytes(t, b"\xc0\xaf") == rep * 2  # overlong
    assert b"".join(t.push([0], [256])) == b"ok"


def test_invalid_bytes_error_policy():
    import lfm2_b200
    t = streams(BYTES)
    with pytest.raises(lfm2_b200.LfmError, match="invalid UTF-8"):
        t.push([0, 0, 0], list(b"a\xffb"))
    t.reset(0)
    assert push_bytes(t, b"\xf0\x9f") == b""
    with pytest.raises(lfm2_b200.LfmError):
        push_bytes(t, b"x")


def test_finish_with_incomplete_sequence():
    import lfm2_b200
    t = streams(BYTES)
    assert push_bytes(t, b"h\xf0\x9f") == b"h"
    with pytest.raises(lfm2_b200.LfmError, match="incomplete"):
        t.finish(0)
    assert t.finish(0) == b""  # finish leaves the stream empty
    assert push_bytes(t, b"k") == b"k"
    r = streams(BYTES, replace=True)
    push_bytes(r, b"\xf0\x9f")
    assert r.finish(0) == "�".encode()
    assert r.finish(0) == b""


def test_multibyte_split_across_tokens_waits():
    t = streams(BYTES)
    for ch in ["é", "日", "🦀", "€"]:
        b = ch.encode()
        for k in range(len(b) - 1):
            assert push_bytes(t, b[k:k + 1]) == b""
        assert push_bytes(t, b[-1:]) == b
    assert t.finish(0) == b""


def xorshift_samples(n, length=120, seed=0x12345678):
    alphabet = [" ", " ", "'", "s", "m", "r", "e", "v", "l", "t", "d", "!", ",", ".", "?", "a", "é", "🦀"]
    state = seed
    out = ["Hello , world ! I 'm fine . We 're ready ?",
           "long prefix to force incremental emission: ' ' ' , . 's 'm 're 've 't 'd 'll",
           "Unicode café 🦀 ' 日本語 , hello ." * 8]
    mask = (1 << 64) - 1
    for _ in range(n):
        s = []
        for _ in range(length):
            state ^= (state << 13) & mask
            state ^= state >> 7
            state ^= (state << 17) & mask
            s.append(alphabet[state % len(alphabet)])
        out.append("".join(s))
    return out


def test_streamed_cleanup_equals_whole_sequence_cleanup():
    """engine/tests/text_stream.rs: one character at a time, and byte pieces
    cut at random boundaries (UTF-8 buffering), give the whole-text cleanup."""
    rng = np.random.default_rng(3)
    for sample in xorshift_samples(200):
        data = sample.encode()
        expected = ref.clean_spaces(data)
        # one character per token
        chars = list(sample)
        pieces = [c.encode() for c in chars]
        t = streams(pieces, clean=True)
        got = b"".join(t.push([0] * len(chars), list(range(len(chars))))) + t.finish(0)
        assert got == expected, sample
        # random byte cuts: pieces end inside multi-byte characters
        cuts = sorted(set(rng.integers(1, len(data), size=len(data) // 3).tolist()))
        parts = [data[a:b] for a, b in zip([0] + cuts, cuts + [len(data)])]
        t = streams(parts, clean=True)
        got = b"".join(t.push([0] * len(parts), list(range(len(parts))))) + t.finish(0)
        assert got == expected, sample


@pytest.mark.parametrize("replace", [False, True])
def test_interleaved_sessions_match_restatement(replace):
    """Several sessions fed in one interleaved token stream (what a batched
    decode step produces) against independent restated decoders."""
    import lfm2_b200
    rng = np.random.default_rng(11 + int(replace))
    vocab = [b"", b" ", b"'", b"s", b"m", b"re", b"ll", b" ,", b" .", b"!", "é".encode(), "🦀".encode()[:2],
             "🦀".encode()[2:], "日".encode()[:1], "日".encode()[1:], b"\xff" if replace else b"z", b"hello", b"?"]
    nsess = 5
    t = streams(vocab, nsess, clean=True, replace=replace)
    us = [ref.Utf8Stream(replace) for _ in range(nsess)]
    dt = [ref.DecodedText(True) for _ in range(nsess)]
    got = [b""] * nsess
    want = [b""] * nsess
    for step in range(300):
        ss = rng.permutation(nsess)[: rng.integers(1, nsess + 1)]
        tok = rng.integers(0, len(vocab), len(ss))
        try:
            outs = t.push(ss.tolist(), tok.tolist())
        except lfm2_b200.LfmError:
            outs = None
        ok = True
        rs = []
        for s, k in zip(ss, tok):
            try:
                rs.append(dt[s].push(us[s].push(vocab[k])))
            except ref.InvalidUtf8:
                ok = False
                break
        assert (outs is not None) == ok
        if not ok:
            return  # the error policy stops at the first invalid sequence (covered above)
        for s, o, r in zip(ss, outs, rs):
            got[s] += o
            want[s] += r
    for s in range(nsess):
        try:
            w = dt[s].finish(us[s].finish())
        except (ref.IncompleteUtf8, ref.InvalidUtf8):
            with pytest.raises(lfm2_b200.LfmError):
                t.finish(s)
            got[s] = want[s] = b""
            continue
        got[s] += t.finish(s)
        want[s] += w
    assert got == want
