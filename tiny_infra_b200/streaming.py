"""Incremental detokenization of a generation stream (the reference's ``consume_stream``,
main.py:12-32): after every token the whole generated sequence is decoded (special tokens
skipped) and only the text past what was already emitted is passed on, so a character that
spans several tokens appears once it is complete."""
from __future__ import annotations

import sys


async def stream_text(stream_gen, tokenizer, skip_special_tokens: bool = True):
    """Yield the new text of each step of ``stream_gen`` (an async iterator of token ids, e.g.
    ``ContinuousBatcher.generate_stream``); ``tokenizer.decode(ids, skip_special_tokens=...)``
    is the only tokenizer call."""
    ids: list[int] = []
    printed = 0
    async for tok in stream_gen:
        ids.append(int(tok))
        text = tokenizer.decode(ids, skip_special_tokens=skip_special_tokens)
        new = text[printed:]
        if new:
            printed = len(text)
            yield new


async def consume_stream(request_id, stream_gen, tokenizer, write=None) -> None:
    """main.py:12-32: print a request's text as it is generated, with the reference's messages;
    an error raised by the stream is reported, not propagated.  ``write`` defaults to
    ``sys.stdout.write``."""
    out = write or sys.stdout.write
    out(f"\n[Request {request_id}] Started streaming....\n")
    try:
        async for new in stream_text(stream_gen, tokenizer):
            out(f"\n[Req {request_id}]: {new}")
            if write is None:
                sys.stdout.flush()
    except Exception as e:  # noqa: BLE001 - the reference reports any stream error
        out(f"\n[Request {request_id}] Error during streaming: {e}\n")
    else:
        out(f"\n[Request {request_id}] Streaming completed.\n")
