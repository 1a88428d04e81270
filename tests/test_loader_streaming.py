"""The reference's checkpoint format (engine/loader.py:34-79) and its streaming consumer
(main.py:12-32), on the host: a tiny checkpoint written with the reference's flat keys maps to
the reference's state-dict names (strict: missing and unexpected keys raise; a tied lm_head
becomes the embedding tensor), and the incremental detokenizer emits each completed piece of
text once, in order, skipping special tokens, and reports a stream error."""
import asyncio

import pytest
import torch

from tiny_infra_b200.loader import read_reference_checkpoint, reference_key_map
from tiny_infra_b200.streaming import consume_stream, stream_text


def _checkpoint(path, layers=2, tied=True, H=16, NH=2, KVH=1, D=8, I=32, V=50, drop=None,
                extra=None):
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(0)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    t = {"token_embeddings": r(V, H), "final_norm_weight": r(H)}
    t["lm_head"] = t["token_embeddings"].clone() if tied else r(V, H)
    for i in range(layers):
        b = f"blocks.{i}"
        t.update({f"{b}.attn.q_proj.weight": r(NH * D, H), f"{b}.attn.q_proj.bias": r(NH * D),
                  f"{b}.attn.k_proj.weight": r(KVH * D, H), f"{b}.attn.k_proj.bias": r(KVH * D),
                  f"{b}.attn.v_proj.weight": r(KVH * D, H), f"{b}.attn.v_proj.bias": r(KVH * D),
                  f"{b}.attn.out_proj.weight": r(H, NH * D), f"{b}.mlp.gate_proj": r(I, H),
                  f"{b}.mlp.up_proj": r(I, H), f"{b}.mlp.down_proj": r(H, I),
                  f"{b}.attn_norm": r(H), f"{b}.mlp_norm": r(H)})
    if drop:
        del t[drop]
    if extra:
        t[extra] = r(3)
    save_file(t, str(path))
    return t


def test_checkpoint_names_map_to_reference_state_dict(tmp_path):
    p = tmp_path / "w.safetensors"
    raw = _checkpoint(p)
    sd = read_reference_checkpoint(str(p), 2)
    m = reference_key_map(2)
    assert set(sd) == set(m.values()) and len(m) == 3 + 2 * 12
    for k, v in m.items():
        assert torch.equal(sd[v], raw[k]), k
    assert sd["model.layers.1.mlp.gate_proj.weight"].shape == (32, 16)
    assert sd["lm_head.weight"] is sd["model.embed_tokens.weight"]       # tied: one buffer
    p2 = tmp_path / "u.safetensors"
    _checkpoint(p2, tied=False)
    sd2 = read_reference_checkpoint(str(p2), 2)
    assert sd2["lm_head.weight"] is not sd2["model.embed_tokens.weight"]


def test_checkpoint_strictness(tmp_path):
    p = tmp_path / "m.safetensors"
    _checkpoint(p, drop="blocks.1.mlp_norm")
    with pytest.raises(KeyError):
        read_reference_checkpoint(str(p), 2)
    p = tmp_path / "x.safetensors"
    _checkpoint(p, extra="blocks.0.attn.rotary")
    with pytest.raises(RuntimeError, match="Unexpected"):
        read_reference_checkpoint(str(p), 2)


class _Tok:
    """ids 1..26 -> a..z, 0 special; 30 followed by 31 is one two-token character."""

    def decode(self, ids, skip_special_tokens=True):
        out, i = [], 0
        while i < len(ids):
            t = ids[i]
            if t == 0:
                if not skip_special_tokens:
                    out.append("<s>")
            elif t == 30:
                if i + 1 < len(ids) and ids[i + 1] == 31:
                    out.append("\u00e9")
                    i += 1
            else:
                out.append(chr(ord("a") + t - 1))
            i += 1
        return "".join(out)


async def _gen(ids, fail_at=None):
    for i, t in enumerate(ids):
        if i == fail_at:
            raise RuntimeError("slot freed")
        yield t


def test_stream_text_emits_completed_text_once():
    async def run():
        return [s async for s in stream_text(_gen([8, 9, 0, 30, 31, 1]), _Tok())]
    assert asyncio.run(run()) == ["h", "i", "\u00e9", "a"]


def test_consume_stream_messages_and_errors():
    out = []
    asyncio.run(consume_stream("r1", _gen([8, 9]), _Tok(), write=out.append))
    text = "".join(out)
    assert "[Request r1] Started streaming" in text and "[Req r1]: h" in text
    assert "[Req r1]: i" in text and "Streaming completed" in text
    out.clear()
    asyncio.run(consume_stream("r2", _gen([8, 9, 1], fail_at=2), _Tok(), write=out.append))
    text = "".join(out)
    assert "Error during streaming: slot freed" in text and "completed" not in text
