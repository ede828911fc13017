"""Python restatement of the reference's streaming text stages (test
infrastructure only: the checker of the engine library's lfm_text_* path).

* `Utf8Stream` restates tokenizer/src/stream.rs:48-131 (push: complete text
  out, an incomplete tail kept, invalid bytes an error or one U+FFFD per
  maximal invalid subsequence; finish: the tail as an error or one U+FFFD).
  Python's UTF-8 decoder reports the same valid prefix and the same maximal
  invalid subsequences as Rust's str::from_utf8 (both follow the Unicode
  "maximal subpart" practice).
* `DecodedText` and `clean_spaces` restate engine/src/text_output.rs:9-106.
"""


class InvalidUtf8(Exception):
    def __init__(self, valid_up_to, data):
        super().__init__(f"invalid UTF-8 after {valid_up_to} bytes")
        self.valid_up_to = valid_up_to
        self.data = data


class IncompleteUtf8(Exception):
    pass


def _from_utf8(b: bytes):
    """(valid_up_to, error_len or None) like Rust's Utf8Error, or None if valid."""
    try:
        b.decode("utf-8")
        return None
    except UnicodeDecodeError as e:
        if e.reason == "unexpected end of data" and e.end == len(b):
            return e.start, None
        return e.start, e.end - e.start


class Utf8Stream:
    def __init__(self, replace: bool):
        self.pending = b""
        self.replace = replace

    def push(self, data: bytes) -> str:
        self.pending += data
        out, consumed = [], 0
        while True:
            rest = self.pending[consumed:]
            err = _from_utf8(rest)
            if err is None:
                out.append(rest.decode("utf-8"))
                consumed = len(self.pending)
                break
            good, bad = err
            out.append(rest[:good].decode("utf-8"))
            if bad is None:
                consumed += good
                break
            if not self.replace:
                raise InvalidUtf8(consumed + good, self.pending)
            out.append("�")
            consumed += good + bad
        self.pending = self.pending[consumed:]
        return "".join(out)

    def finish(self) -> str:
        if not self.pending:
            return ""
        pending, self.pending = self.pending, b""
        if self.replace:
            return "�"
        err = _from_utf8(pending)
        if err is None:
            return pending.decode("utf-8")
        if err[1] is not None:
            raise InvalidUtf8(err[0], pending)
        raise IncompleteUtf8()


def clean_spaces(text: bytes) -> bytes:
    """text_output.rs:59-106 (the tokenizer decoder's in-place passes)."""
    t = bytearray(text)
    total = len(t)
    total1 = total
    total = 1 if total > 0 else 0
    for i in range(1, total1):
        x = t[i]
        if t[i - 1] == 0x20 and x in b"?!.,":
            total -= 1
        t[total] = x
        total += 1
    total2 = total
    total = 1 if total > 0 else 0
    i = 1
    while i < total2:
        x = t[i]
        if x == 0x27 and i + 1 < total2 and t[i - 1] == 0x20 and t[i + 1] == 0x20:
            total -= 1
            i += 1
            t[i] = 0
        t[total] = x
        total += 1
        i += 1
    total3 = total
    total = 1 if total > 0 else 0
    for i in range(1, total3):
        x = t[i]
        if t[i - 1] == 0x20 and x == 0x27 and i + 1 < total3:
            x1 = t[i + 1]
            if x1 in b"td":
                pass
            elif x1 in b"sm":
                total -= 1
            elif i + 2 < total3:
                x2 = t[i + 2]
                if x1 == ord("l") and x2 == ord("l"):
                    pass
                elif (x1 == ord("r") and x2 == ord("e")) or (x1 == ord("v") and x2 == ord("e")):
                    total -= 1
        t[total] = x
        total += 1
    return bytes(t[:total])


class DecodedText:
    """text_output.rs:9-53."""

    def __init__(self, clean: bool):
        self.raw = b""
        self.emitted = b""
        self.clean = clean

    def push(self, chunk: str) -> bytes:
        self.raw += chunk.encode("utf-8")
        return self._take(False)

    def finish(self, chunk: str) -> bytes:
        self.raw += chunk.encode("utf-8")
        return self._take(True)

    def _take(self, final: bool) -> bytes:
        text = clean_spaces(self.raw) if self.clean else self.raw
        end = len(text) if (final or not self.clean) else max(len(text) - 16, 0)
        while 0 < end < len(text) and (text[end] & 0xC0) == 0x80:
            end -= 1
        assert text.startswith(self.emitted), "cleanup changed an already-emitted prefix"
        end = max(end, len(self.emitted))
        delta = text[len(self.emitted):end]
        self.emitted += delta
        return delta
