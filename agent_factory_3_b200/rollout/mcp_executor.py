"""Tool execution and tool/prompt discovery over MCP clients (reference:
rollout/mcp_executor.py:21-358).

* Namespaces are the keys of the MCP config; namespaces starting with ``builtin_`` or
  ``system_`` go into the system message, the rest into the developer message.
* Tool schemas are trimmed into harmony's JSON-schema variant (no titles, null defaults
  dropped, ``anyOf`` collapsed to a type list); tools whose annotations say
  ``include_in_prompt=False`` are hidden when filtering is on; descriptions can be overridden
  per namespace.
* A call ``namespace.tool`` (or a builtin short name like ``python``) receives JSON arguments;
  a raw string is mapped to the schema's ``rawStringParam`` or to the single required string
  parameter.  Timeouts and exceptions become error reports, never exceptions.
  ``structured_content.early_exit`` ends the episode.
* ``{{mcp_prompt:ns.name}}`` in prompt text is replaced by the server's prompt.
"""
from __future__ import annotations

import copy
import json
import logging
import re
import time
from typing import Any, Optional

from pydantic import BaseModel

from .harmony import ToolDescription
from .types import ToolErrorType

logger = logging.getLogger(__name__)

SYSTEM_NAMESPACE_PREFIXES = ("builtin_", "system_")


def is_system_namespace(namespace: str) -> bool:
    return namespace.startswith(SYSTEM_NAMESPACE_PREFIXES)


class ToolMetadata(BaseModel):
    namespace: str
    name: str
    raw_string_param: Optional[str] = None
    input_schema: Optional[dict[str, Any]] = None


class ToolNamespaceConfig(BaseModel):
    name: str
    description: Optional[str] = None
    tools: list[Any] = []


class ToolCallReport(BaseModel):
    tool_name: str
    tool_input: str
    tool_output: str
    elapsed: float
    error: Optional[ToolErrorType] = None
    early_exit: bool = False
    structured_output: Optional[dict[str, Any]] = None


class McpExecutorError(Exception):
    pass


class McpExecutor:
    def __init__(self, clients: dict | None, tool_call_timeout: float = 60.0,
                 filter_by_include_in_prompt: bool = True,
                 description_overrides: dict | None = None):
        self.clients = clients or {}
        self.tool_call_timeout = tool_call_timeout
        self.filter_by_include_in_prompt = filter_by_include_in_prompt
        self._tool_metadata: dict[str, ToolMetadata] = {}
        self._description_overrides = description_overrides or {}

    @property
    def has_clients(self) -> bool:
        return bool(self.clients)

    @staticmethod
    def trim_schema(schema: dict) -> dict:
        schema = dict(schema)
        schema.pop("title", None)
        if "default" in schema and schema["default"] is None:
            del schema["default"]
        if "anyOf" in schema:
            types = [t["type"] for t in schema["anyOf"] if "type" in t and t["type"] != "null"]
            if types:
                schema["type"] = types if len(types) > 1 else types[0]
            del schema["anyOf"]
        if "properties" in schema:
            schema["properties"] = {k: McpExecutor.trim_schema(v) for k, v in schema["properties"].items()}
        return schema

    def _visible(self, tool) -> bool:
        if not self.filter_by_include_in_prompt:
            return True
        ann = getattr(tool, "annotations", None)
        if ann is None:
            return True
        inc = getattr(ann, "include_in_prompt", None)
        if inc is None and hasattr(ann, "model_extra") and ann.model_extra:
            inc = ann.model_extra.get("include_in_prompt")
        return True if inc is None else bool(inc)

    async def get_tool_configs(self) -> list[ToolNamespaceConfig]:
        out = []
        for ns, client in self.clients.items():
            ov = self._description_overrides.get(ns, {})
            tool_ov = ov.get("tools", {})
            instr = ov.get("instructions")
            if instr is None:
                ir = getattr(client, "initialize_result", None)
                instr = getattr(ir, "instructions", None)
            tools = []
            for t in await client.list_tools():
                if not self._visible(t):
                    continue
                schema = self.trim_schema(copy.deepcopy(t.inputSchema or {}))
                key = f"{ns}.{t.name}"
                self._tool_metadata[key] = ToolMetadata(
                    namespace=ns, name=t.name, raw_string_param=self._raw_string_param(schema),
                    input_schema=schema)
                tools.append(ToolDescription(name=t.name, description=tool_ov.get(t.name, t.description or ""),
                                             parameters=schema))
            out.append(ToolNamespaceConfig(name=ns, description=instr, tools=tools))
        return out

    @staticmethod
    def _raw_string_param(schema: dict) -> Optional[str]:
        for name, ps in (schema.get("properties") or {}).items():
            if ps.get("rawStringParam"):
                return name
        return None

    def _single_string_param(self, key: str) -> Optional[str]:
        md = self._tool_metadata.get(key)
        if not md or not md.input_schema:
            return None
        req = set(md.input_schema.get("required") or [])
        if len(req) != 1:
            return None
        name = next(iter(req))
        return name if (md.input_schema.get("properties") or {}).get(name, {}).get("type") == "string" else None

    def resolve_reference(self, ref: str) -> tuple[str, str]:
        if "." in ref:
            ns, name = ref.split(".", 1)
            return ns, name
        for ns in self.clients:
            if is_system_namespace(ns) and ns.endswith(f"_{ref}"):
                return ns, ref
        raise ValueError(f"Unknown tool reference: {ref}")

    def prepare_args(self, ns: str, name: str, content: str) -> dict:
        key = f"{ns}.{name}"
        md = self._tool_metadata.get(key)
        if md and md.raw_string_param:
            try:
                parsed = json.loads(content) if content else None
            except json.JSONDecodeError:
                parsed = None
            if isinstance(parsed, dict):
                return parsed
            return {md.raw_string_param: content}
        if not content:
            return {}
        try:
            parsed = json.loads(content)
        except json.JSONDecodeError:
            parsed = None
        if isinstance(parsed, dict):
            return parsed
        single = self._single_string_param(key)
        if single:
            return {single: content}
        raise ValueError(f"Tool {key} received non-JSON input and has no single string parameter")

    async def call_tool(self, recipient: str, content: str) -> ToolCallReport:
        start = time.perf_counter()
        tool_name = recipient
        try:
            ns, tool_name = self.resolve_reference(recipient)
            if ns not in self.clients:
                raise ValueError(f"Unknown tool namespace: {recipient}")
            args = self.prepare_args(ns, tool_name, content)
            res = await self.clients[ns].call_tool(tool_name, arguments=args,
                                                   timeout=self.tool_call_timeout)
            texts = [b.text for b in res.content if getattr(b, "type", "") == "text"]
            structured = getattr(res, "structuredContent", None) or getattr(res, "structured_content", None) or {}
            if isinstance(structured, dict) and "result" in structured and len(structured) == 1 \
                    and isinstance(structured["result"], dict):
                structured = structured["result"]
            if not structured:
                # a fenced ```metadata``` JSON text block (servers that mix text and images)
                for t in texts:
                    st = t.strip()
                    if st.startswith("```metadata") and st.endswith("```"):
                        try:
                            parsed = json.loads(st[len("```metadata"):-3])
                            structured = parsed if isinstance(parsed, dict) else {}
                        except ValueError:
                            pass
            if not structured and len(texts) == 1:
                # servers that return a JSON object only as text: treat it as structured
                try:
                    parsed = json.loads(texts[0])
                    structured = parsed if isinstance(parsed, dict) else {}
                except json.JSONDecodeError:
                    structured = {}
            return ToolCallReport(
                tool_name=tool_name, tool_input=content,
                tool_output="\n".join(texts) if texts else "<no text output>",
                elapsed=time.perf_counter() - start,
                error=ToolErrorType.TOOL_ERROR if getattr(res, "isError", False) else None,
                early_exit=bool(structured.get("early_exit", False)) if isinstance(structured, dict) else False,
                structured_output=structured or None)
        except (TimeoutError, __import__("asyncio").TimeoutError):
            return ToolCallReport(tool_name=tool_name, tool_input=content,
                                  tool_output="Tool execution timed out.",
                                  elapsed=time.perf_counter() - start, error=ToolErrorType.TIMEOUT)
        except Exception as exc:  # noqa: BLE001
            return ToolCallReport(tool_name=tool_name, tool_input=content, tool_output=str(exc),
                                  elapsed=time.perf_counter() - start,
                                  error=ToolErrorType.EXCEPTION)

    async def get_prompt(self, reference: str) -> str:
        if not self.clients:
            raise McpExecutorError(f"Prompt '{reference}' requested but no MCP client configured.")
        ns, name = self.resolve_reference(reference)
        p = await self.clients[ns].get_prompt(name)
        return p.messages[0].content.text

    async def resolve_prompts(self, text: str, strict: bool = False) -> str:
        if not self.clients or not text:
            return text
        for name in set(re.findall(r"\{\{mcp_prompt:([^}]+)\}\}", text)):
            try:
                text = text.replace(f"{{{{mcp_prompt:{name}}}}}", await self.get_prompt(name))
            except Exception as e:  # noqa: BLE001
                if strict:
                    raise
                logger.warning("failed to load MCP prompt %r: %s", name, e)
        return text
