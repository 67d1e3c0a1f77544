"""Chat templating of corpus rows into spans with explicit supervision flags.

A corpus row holds ``segments`` (text or image) and a ``format``. ``build(row)`` returns
``(spans, direction, opens_with_bos)`` (reference ``data/chat.py:1-182``):

* ``caption`` rows whose stored order is text→image (T2I) or image→text (I2T) become one user
  turn and one assistant turn in Qwen chat form (``<|im_start|>role\\n … <|im_end|>\\n``);
  the instruction of the user turn is picked from a fixed list by hashing the sample id, so a
  resumed run rebuilds the same text;
* ``conversation`` / ``text_conversation`` rows keep their turns, one message per (role, turn);
* everything else stays a natural document (no chat wrapper, no opening ``<|im_start|>``).

Supervision: corpus text is supervised (user turns included: this is pretraining, not SFT);
text that the template fabricates (role headers, instructions) is neither supervised nor
counted as corpus tokens; the ``<|im_end|>`` closer is supervised (the model learns to stop)
but not counted. The packer's document BOS plays the first ``<|im_start|>``, so the first
header carries only the role name. No thinking prefix is emitted.
"""

from __future__ import annotations

import hashlib

# The instruction only marks the direction of the turn; the corpus text carries the content.
# Several plain phrasings keep the model from tying a direction to one literal string.
T2I_PROMPTS = (
    "Create a picture of: ",
    "Paint this scene: ",
    "Generate an image showing the following. ",
    "Please draw what this text describes: ",
    "Render a photo for this caption: ",
    "Make a picture that fits this description: ",
    "Show this as an image: ",
    "Picture the following and generate it: ",
    "Turn this text into an image: ",
    "I would like an image of the following: ",
    "Depict the following in an image: ",
    "Image request: ",
)

I2T_PROMPTS = (
    "What is in this picture?",
    "Describe the image.",
    "Write a caption for the picture above.",
    "What does this photo show?",
    "Explain what you see here.",
    "Give a description of this picture.",
    "Caption this.",
    "Summarise the image in words.",
    "What can you see in the image?",
    "Tell me about this picture.",
    "Describe what is happening in the image.",
    "Provide a caption.",
)

IM_START = "<|im_start|>"
IM_END = "<|im_end|>\n"
USER = "user\n"
ASSISTANT = "assistant\n"


def pick(options, sample_id, salt):
    """Deterministic choice from ``options`` keyed by the immutable sample id."""
    digest = hashlib.sha256(f"{salt}|{sample_id}".encode()).digest()
    return options[int.from_bytes(digest[:8], "little") % len(options)]


def text_span(value, supervised, synthetic):
    return dict(kind="text", text=value, supervised=supervised, synthetic=synthetic)


def corpus_text(value):
    """Text from the corpus: supervised and counted."""
    return text_span(value, True, False)


def template_text(value):
    """Text made up by the template: neither supervised nor counted."""
    return text_span(value, False, True)


def end_of_turn():
    """``<|im_end|>``: supervised so the model learns to stop, not counted as corpus."""
    return text_span(IM_END, True, True)


def image_span(index, role=None):
    span = dict(kind="image", image_index=index)
    if role is not None:
        span["role"] = role
    return span


def role_header(role, first):
    # the packer's BOS is the first <|im_start|>
    return template_text(role if first else IM_START + role)


def caption_direction(segments):
    """``T2I`` for stored order text→image, ``I2T`` for image→text, else ``None``."""
    kinds = tuple(s["kind"] for s in segments)
    return {("text", "image"): "T2I", ("image", "text"): "I2T"}.get(kinds)


def caption_spans(segments, direction, sample_id):
    body = next(s for s in segments if s["kind"] == "text")["text"]
    picture = next(s for s in segments if s["kind"] == "image")["image_index"]
    spans = [role_header(USER, True)]
    if direction == "T2I":
        spans += [template_text(pick(T2I_PROMPTS, sample_id, "t2i")), corpus_text(body), end_of_turn(),
                  role_header(ASSISTANT, False), image_span(picture)]
    else:
        spans += [image_span(picture), template_text(pick(I2T_PROMPTS, sample_id, "i2t")), end_of_turn(),
                  role_header(ASSISTANT, False), corpus_text(body)]
    spans.append(end_of_turn())
    return spans


def conversation_spans(segments):
    """One message per consecutive (role, turn) group; a missing role means the user."""
    spans, current = [], None
    for segment in segments:
        role = segment.get("role") or "user"
        key = (role, segment.get("turn"))
        if key != current:
            if current is not None:
                spans.append(end_of_turn())
            spans.append(role_header(ASSISTANT if role == "assistant" else USER, current is None))
            current = key
        if segment["kind"] == "image":
            spans.append(image_span(segment["image_index"], role))
        elif segment.get("text"):
            spans.append(corpus_text(segment["text"]))
    if current is not None:
        spans.append(end_of_turn())
    return spans


def natural_spans(segments):
    """Interleaved documents keep their natural form."""
    out = []
    for s in segments:
        if s["kind"] == "image":
            out.append(image_span(s["image_index"]))
        elif s.get("text"):
            out.append(corpus_text(s["text"]))
    return out


def build(row):
    """``(spans, direction, opens_with_bos)`` for one corpus row (see the module docstring)."""
    segments, fmt = row["segments"], row.get("format")
    if fmt == "caption":
        direction = caption_direction(segments)
        if direction is None:
            return natural_spans(segments), None, False
        return caption_spans(segments, direction, row["sample_id"]), direction, True
    if fmt in ("conversation", "text_conversation"):
        roles = [s.get("role") or "user" for s in segments if s["kind"] == "image"]
        direction = None
        if roles:
            direction = "T2I" if "assistant" in roles else "I2T"
        return conversation_spans(segments), direction, True
    return natural_spans(segments), None, False


def tokenize_spans(spans, encode):
    """Flatten spans to ``(ids, supervised, counted)`` lists with ``encode(text) -> list[int]``.

    Image spans become a ``None`` placeholder id; the packer expands them into visual tokens.
    """
    ids, supervised, counted = [], [], []
    for span in spans:
        if span["kind"] == "image":
            ids.append(None)
            supervised.append(False)
            counted.append(False)
            continue
        toks = list(encode(span["text"]))
        ids += toks
        supervised += [span["supervised"]] * len(toks)
        counted += [not span["synthetic"]] * len(toks)
    return ids, supervised, counted


def row_document(row, encode, visual=None):
    """A raw corpus row (``segments``) -> a packer document (``elements``).

    Consecutive text spans with the same supervision flag merge into one text element
    (``input_ids`` from ``encode``, ``supervised`` flag); image spans become the element that
    ``visual(segment, row)`` returns (default: the stored image segment). The image-loss
    permission of the row and the image entry decides whether the visual may be a generation
    target.
    """
    from .permissions import image_loss_allowed
    spans, direction, opens = build(row)
    images = {s["image_index"]: s for s in row["segments"] if s["kind"] == "image"}
    elements, pending, flag = [], [], None

    def flush():
        nonlocal pending
        if pending:
            elements.append(dict(type="text", input_ids=[i for ids in pending for i in ids], supervised=flag))
            pending = []

    for span in spans:
        if span["kind"] == "image":
            flush()
            segment = images[span["image_index"]]
            element = dict(visual(segment, row) if visual else segment)
            element.setdefault("type", "image")
            element["loss_allowed"] = image_loss_allowed(row, segment)
            elements.append(element)
            continue
        if pending and span["supervised"] != flag:
            flush()
        flag = span["supervised"]
        pending.append(list(encode(span["text"])))
    flush()
    return dict(id=row["sample_id"], elements=elements, direction=direction, templated=opens,
                format=row.get("format"))
