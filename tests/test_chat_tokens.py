"""Chat templating, the token contract and image-loss permissions (CPU)."""

import json

import pytest

from cq_pretrain_b200.config import tiny_config
from cq_pretrain_b200.data import chat, permissions, tokens


def test_caption_templating_and_supervision():
    row = dict(sample_id="s1", format="caption",
               segments=[dict(kind="text", text="a red bus"), dict(kind="image", image_index=0)])
    spans, direction, opens = chat.build(row)
    assert direction == "T2I" and opens
    kinds = [(s["kind"], s.get("supervised"), s.get("synthetic")) for s in spans]
    # header (user, no <|im_start|>: the packer's BOS), instruction, corpus, end, header, image, end
    assert kinds == [("text", False, True), ("text", False, True), ("text", True, False), ("text", True, True),
                     ("text", False, True), ("image", None, None), ("text", True, True)]
    assert spans[0]["text"] == "user\n" and spans[4]["text"] == "<|im_start|>assistant\n"
    assert spans[1]["text"] in chat.T2I_PROMPTS
    again, _, _ = chat.build(row)
    assert again == spans   # deterministic instruction


def test_i2t_conversation_and_natural():
    row = dict(sample_id="x", format="caption",
               segments=[dict(kind="image", image_index=3), dict(kind="text", text="a cat")])
    spans, direction, _ = chat.build(row)
    assert direction == "I2T" and spans[1]["kind"] == "image" and spans[2]["text"] in chat.I2T_PROMPTS
    conv = dict(sample_id="c", format="conversation", segments=[
        dict(kind="text", text="hi", role="user", turn=0), dict(kind="text", text="hello", role="assistant", turn=1),
        dict(kind="image", image_index=0, role="assistant", turn=1)])
    spans, direction, opens = chat.build(conv)
    assert direction == "T2I" and opens
    assert [s["text"] for s in spans if s["kind"] == "text"] == [
        "user\n", "hi", "<|im_end|>\n", "<|im_start|>assistant\n", "hello", "<|im_end|>\n"]
    natural = dict(sample_id="n", format="interleaved",
                   segments=[dict(kind="text", text="x"), dict(kind="image", image_index=0), dict(kind="text", text="")])
    spans, direction, opens = chat.build(natural)
    assert direction is None and not opens and len(spans) == 2


def test_row_document_merges_spans_and_applies_permissions():
    row = dict(sample_id="s2", format="caption", image_loss_allowed=True,
               segments=[dict(kind="text", text="ab"), dict(kind="image", image_index=0, dcvlm_image_loss_allowed=False)])
    doc = chat.row_document(row, encode=lambda text: [ord(c) for c in text])
    kinds = [(e["type"], e.get("supervised")) for e in doc["elements"]]
    assert kinds[0] == ("text", False) and ("image", None) in kinds
    image = next(e for e in doc["elements"] if e["type"] == "image")
    assert image["loss_allowed"] is False and doc["templated"] and doc["direction"] == "T2I"
    supervised = [e for e in doc["elements"] if e["type"] == "text" and e["supervised"]]
    assert [ord("a"), ord("b")] == supervised[0]["input_ids"][:2]


def test_image_loss_permissions_are_strict():
    assert permissions.image_loss_allowed({}, {"image_loss_allowed": True})
    assert not permissions.image_loss_allowed({"image_loss_allowed": True}, {"dcvlm_image_loss_allowed": False})
    for bad in (None, 1, "true"):
        with pytest.raises(ValueError):
            permissions.image_loss_allowed({"image_loss_allowed": False}, {"dcvlm_image_loss_allowed": bad})


def test_token_contract(tmp_path):
    cfg = tiny_config()
    decoder = {str(i): dict(content=t, special=True) for i, t in enumerate(
        ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<|vision_start|>", "<|vision_end|>", "<|image_pad|>",
         "<|fim_pad|>"], start=900)}
    (tmp_path / "tokenizer_config.json").write_text(json.dumps(dict(added_tokens_decoder=decoder)))
    (tmp_path / "tokenizer.json").write_text("{}")
    ids = tokens.token_contract(tmp_path, cfg)
    assert ids["bos"] == 901 and ids["eos"] == 900 and ids["image"] == 905 and ids["text_mask"] == 906
    assert cfg.image_mask_token_id == 905 and cfg.text_mask_token_id == 906
    meta = tokens.tokenizer_metadata(tmp_path)
    assert set(meta["files"]) == {"tokenizer.json", "tokenizer_config.json"}
    assert meta["counting"]["exclude_special_token_ids"][0] == 900
    (tmp_path / "tokenizer.json").write_text("{} ")
    with pytest.raises(ValueError, match="checksum"):
        tokens.tokenizer_metadata(tmp_path, expected=meta)
    cfg.vocab_size = 900
    with pytest.raises(ValueError, match="vocabulary"):
        tokens.token_contract(tmp_path, cfg)
