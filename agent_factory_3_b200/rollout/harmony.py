"""The harmony chat format of gpt-oss: messages, rendering to tokens and parsing of completions.

Token-level layout (one message):
    <|start|>{role}[ to={recipient}][<|channel|>{channel}][ <|constrain|>{type}]<|message|>{text}{end}
with end = <|end|>, <|call|> (assistant tool call) or <|return|> (assistant final answer).
The special-token ids are those of the o200k_harmony vocabulary (201088 entries), so token
streams are interchangeable with the real encoding.  Ordinary text goes through a pluggable
``Tokenizer``: the real o200k_harmony BPE through ``openai_harmony`` when its vocabulary file
is available, else a byte-level tokenizer that maps UTF-8 bytes to ids 0..255 (used offline and
in tests; the model vocabulary is unchanged).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Iterable, Protocol

START, END, MESSAGE, CHANNEL, CONSTRAIN, RETURN, CALL = (200006, 200007, 200008, 200005,
                                                         200003, 200002, 200012)
ENDOFTEXT, STARTOFTEXT = 199999, 199998
SPECIAL_NAMES = {START: "<|start|>", END: "<|end|>", MESSAGE: "<|message|>", CHANNEL: "<|channel|>",
                 CONSTRAIN: "<|constrain|>", RETURN: "<|return|>", CALL: "<|call|>",
                 ENDOFTEXT: "<|endoftext|>", STARTOFTEXT: "<|startoftext|>"}
STOP_TOKENS_ASSISTANT_ACTIONS = [RETURN, CALL]          # generation stops on these
STOP_TOKENS_ALL = [RETURN, CALL, END]


class Tokenizer(Protocol):
    def encode(self, text: str) -> list[int]: ...
    def decode(self, ids: Iterable[int]) -> str: ...


class ByteTokenizer:
    """UTF-8 bytes -> ids 0..255; special ids decode to their names."""

    def encode(self, text: str) -> list[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids: Iterable[int]) -> str:
        out = bytearray()
        parts = []
        for t in ids:
            t = int(t)
            if t < 256:
                out.append(t)
            else:
                if out:
                    parts.append(out.decode("utf-8", errors="replace"))
                    out = bytearray()
                parts.append(SPECIAL_NAMES.get(t, f"<|tok{t}|>"))
        if out:
            parts.append(out.decode("utf-8", errors="replace"))
        return "".join(parts)


class HarmonyBPETokenizer:
    """Adapter over openai_harmony's o200k_harmony encoding (needs its vocabulary file)."""

    def __init__(self):
        from openai_harmony import HarmonyEncodingName, load_harmony_encoding

        self.enc = load_harmony_encoding(HarmonyEncodingName.HARMONY_GPT_OSS)

    def encode(self, text: str) -> list[int]:
        return list(self.enc.encode(text, allowed_special="all"))

    def decode(self, ids: Iterable[int]) -> str:
        return self.enc.decode_utf8(list(ids))


_DEFAULT: Tokenizer | None = None


def default_tokenizer() -> Tokenizer:
    global _DEFAULT
    if _DEFAULT is None:
        try:
            _DEFAULT = HarmonyBPETokenizer()
        except Exception:  # noqa: BLE001 - vocabulary not available offline
            _DEFAULT = ByteTokenizer()
    return _DEFAULT


def set_default_tokenizer(tok: Tokenizer) -> None:
    global _DEFAULT
    _DEFAULT = tok


class Role(str, Enum):
    SYSTEM = "system"
    DEVELOPER = "developer"
    USER = "user"
    ASSISTANT = "assistant"
    TOOL = "tool"


@dataclass
class ToolDescription:
    name: str
    description: str = ""
    parameters: dict | None = None

    def to_dict(self):
        return {"name": self.name, "description": self.description, "parameters": self.parameters}


@dataclass
class Message:
    role: str                       # system / developer / user / assistant / "<namespace.tool>"
    content: str
    channel: str | None = None
    recipient: str | None = None
    content_type: str | None = None  # e.g. "json" (rendered as <|constrain|>json)
    end: int = END                   # END / CALL / RETURN

    @classmethod
    def from_role_and_content(cls, role: str | Role, content: str) -> "Message":
        return cls(role=role.value if isinstance(role, Role) else role, content=content)

    def with_channel(self, ch: str) -> "Message":
        self.channel = ch
        return self

    def with_recipient(self, r: str) -> "Message":
        self.recipient = r
        return self

    def to_dict(self) -> dict:
        return {"role": self.role, "content": self.content, "channel": self.channel,
                "recipient": self.recipient, "content_type": self.content_type, "end": self.end}

    @classmethod
    def from_dict(cls, d: dict) -> "Message":
        return cls(**d)


@dataclass
class Conversation:
    messages: list[Message] = field(default_factory=list)

    @classmethod
    def from_messages(cls, msgs: list[Message]) -> "Conversation":
        return cls(list(msgs))

    def to_dict(self) -> dict:
        return {"messages": [m.to_dict() for m in self.messages]}

    @classmethod
    def from_dict(cls, d: dict) -> "Conversation":
        return cls([Message.from_dict(m) for m in d.get("messages", [])])

    def to_json(self) -> str:
        return json.dumps(self.to_dict())


# ------------------------------------------------------------------ system / developer text
def system_text(model_identity: str, reasoning_effort: str, conversation_start_date: str | None,
                builtin_tools: dict[str, list[ToolDescription]] | None = None) -> str:
    lines = [model_identity, "Knowledge cutoff: 2024-06"]
    if conversation_start_date:
        lines.append(f"Current date: {conversation_start_date}")
    lines.append("")
    lines.append(f"Reasoning: {reasoning_effort}")
    if builtin_tools:
        lines.append("")
        lines.append("# Tools")
        for ns, tools in builtin_tools.items():
            lines.append("")
            lines.append(f"## {ns}")
            if ns != "python":
                lines.append("")
                lines.append(render_namespace(ns, tools))
    lines.append("")
    lines.append("# Valid channels: analysis, commentary, final. Channel must be included for every message.")
    lines.append("Calls to these tools must go to the commentary channel: 'functions'.")
    return "\n".join(lines)


def _ts_type(schema: dict | None) -> str:
    if not schema:
        return "any"
    t = schema.get("type")
    if "enum" in schema:
        return " | ".join(json.dumps(v) for v in schema["enum"])
    if t == "string":
        return "string"
    if t in ("integer", "number"):
        return "number"
    if t == "boolean":
        return "boolean"
    if t == "array":
        return f"{_ts_type(schema.get('items'))}[]"
    if t == "object":
        props = schema.get("properties") or {}
        req = set(schema.get("required") or [])
        inner = ", ".join(f"{k}{'' if k in req else '?'}: {_ts_type(v)}" for k, v in props.items())
        return "{" + inner + "}"
    return "any"


def render_namespace(namespace: str, tools: list[ToolDescription]) -> str:
    """TypeScript-style tool declarations used by harmony developer/system messages."""
    out = [f"namespace {namespace} {{", ""]
    for t in tools:
        if t.description:
            for line in t.description.strip().splitlines():
                out.append(f"// {line}")
        params = t.parameters or {}
        props = params.get("properties") or {}
        if props:
            req = set(params.get("required") or [])
            out.append(f"type {t.name} = (_: {{")
            for k, v in props.items():
                if v.get("description"):
                    out.append(f"// {v['description']}")
                default = f" // default: {json.dumps(v['default'])}" if "default" in v else ""
                out.append(f"{k}{'' if k in req else '?'}: {_ts_type(v)},{default}")
            out.append("}) => any;")
        else:
            out.append(f"type {t.name} = () => any;")
        out.append("")
    out.append(f"}} // namespace {namespace}")
    return "\n".join(out)


def developer_text(instructions: str | None, function_tools: dict[str, list[ToolDescription]]) -> str:
    parts = []
    if instructions:
        parts.append("# Instructions\n\n" + instructions)
    if function_tools:
        tool_lines = ["# Tools"]
        for ns, tools in function_tools.items():
            tool_lines.append("")
            tool_lines.append(f"## {ns}")
            tool_lines.append("")
            tool_lines.append(render_namespace(ns, tools))
        parts.append("\n".join(tool_lines))
    return "\n\n".join(parts)


# ------------------------------------------------------------------ encoding
class HarmonyEncoding:
    def __init__(self, tokenizer: Tokenizer | None = None):
        self.tok = tokenizer or default_tokenizer()

    def stop_tokens_for_assistant_actions(self) -> list[int]:
        return list(STOP_TOKENS_ASSISTANT_ACTIONS)

    def render_header(self, m: Message) -> list[int]:
        ids = [START] + self.tok.encode(m.role)
        if m.recipient and m.role != Role.ASSISTANT.value:
            ids += self.tok.encode(f" to={m.recipient}")
        if m.channel:
            ids += [CHANNEL] + self.tok.encode(m.channel)
        if m.recipient and m.role == Role.ASSISTANT.value:
            ids += self.tok.encode(f" to={m.recipient}")
        if m.content_type:
            ids += self.tok.encode(" ") + [CONSTRAIN] + self.tok.encode(m.content_type)
        return ids + [MESSAGE]

    def render(self, m: Message) -> list[int]:
        return self.render_header(m) + self.tok.encode(m.content) + [m.end]

    def render_conversation_for_completion(self, conv: Conversation, next_role: str = "assistant",
                                           auto_drop_analysis: bool = True) -> list[int]:
        msgs = conv.messages
        if auto_drop_analysis:
            # analysis messages before the last final answer are dropped (harmony convention)
            last_final = max((i for i, m in enumerate(msgs)
                              if m.role == "assistant" and m.channel == "final"), default=-1)
            msgs = [m for i, m in enumerate(msgs)
                    if not (i < last_final and m.role == "assistant" and m.channel == "analysis")]
        ids: list[int] = []
        for m in msgs:
            ids += self.render(m)
        return ids + [START] + self.tok.encode(next_role)

    def render_conversation(self, conv: Conversation) -> list[int]:
        ids: list[int] = []
        for m in conv.messages:
            ids += self.render(m)
        return ids

    def decode(self, ids: Iterable[int]) -> str:
        return self.tok.decode(ids)

    def parse_messages_from_completion_tokens(self, ids: list[int], role: str = "assistant",
                                              strict: bool = True) -> list[Message]:
        """Parse tokens generated after ``<|start|>{role}``; a completion may contain several
        messages, each introduced by <|start|>.  Raises ValueError on malformed input when
        ``strict``."""
        msgs: list[Message] = []
        i = 0
        cur_role = role
        n = len(ids)
        while i < n:
            # header: text up to <|message|>
            try:
                mpos = ids.index(MESSAGE, i)
            except ValueError:
                if strict:
                    raise ValueError("harmony parse: missing <|message|>") from None
                break
            header = ids[i:mpos]
            # end token
            j = mpos + 1
            while j < n and ids[j] not in (END, CALL, RETURN):
                if ids[j] == START:
                    if strict:
                        raise ValueError("harmony parse: <|start|> inside message content")
                    break
                j += 1
            if j >= n and strict:
                raise ValueError("harmony parse: message is not terminated")
            end_tok = ids[j] if j < n else END
            content = self.tok.decode(ids[mpos + 1:j])
            channel = recipient = ctype = None
            seg = []
            hdr_parts = []
            for t in header:
                if t in (CHANNEL, CONSTRAIN):
                    hdr_parts.append(("txt", self.tok.decode(seg)))
                    seg = []
                    hdr_parts.append(("sp", t))
                else:
                    seg.append(t)
            hdr_parts.append(("txt", self.tok.decode(seg)))
            head_text = hdr_parts[0][1] if hdr_parts else ""
            k = 1
            while k < len(hdr_parts):
                kind, val = hdr_parts[k]
                if kind == "sp":
                    nxt = hdr_parts[k + 1][1] if k + 1 < len(hdr_parts) else ""
                    if val == CHANNEL:
                        toks = nxt.split()
                        channel = toks[0] if toks else ""
                        for tkn in toks[1:]:
                            if tkn.startswith("to="):
                                recipient = tkn[3:]
                    else:
                        ctype = nxt.strip()
                    k += 2
                else:
                    k += 1
            words = head_text.split()
            r = cur_role
            if msgs and words and not words[0].startswith("to="):
                r = words[0]  # later messages repeat the role after their <|start|>
            for w in words:
                if w.startswith("to="):
                    recipient = w[3:]
            msgs.append(Message(role=r, content=content, channel=channel, recipient=recipient,
                                content_type=ctype, end=end_tok))
            i = j + 1
            if i < n and ids[i] == START:
                i += 1
            elif i < n and strict:
                raise ValueError("harmony parse: expected <|start|> between messages")
        return msgs


class StreamableParser:
    """Incremental header tracker for segment-aware sampling: reports whether the generated
    prefix is still in the header (before <|message|>) and the channel/recipient once known."""

    def __init__(self, encoding: HarmonyEncoding):
        self.enc = encoding
        self.tokens: list[int] = []

    def process(self, t: int) -> None:
        self.tokens.append(int(t))

    @property
    def in_header(self) -> bool:
        return MESSAGE not in self.tokens

    def header_fields(self) -> tuple[str | None, str | None]:
        if self.in_header:
            return None, None
        hdr = self.tokens[: self.tokens.index(MESSAGE)]
        text = self.enc.tok.decode([t for t in hdr if t not in (CHANNEL, CONSTRAIN)])
        channel = recipient = None
        if CHANNEL in hdr:
            after = self.enc.tok.decode(hdr[hdr.index(CHANNEL) + 1:])
            w = after.split()
            channel = w[0] if w else None
        for w in text.split():
            if w.startswith("to="):
                recipient = w[3:]
        return channel, recipient
