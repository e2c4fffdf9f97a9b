"""Initial harmony conversation of a rollout (reference: rollout/conversation_builder.py:19-135):
system message (identity, date, reasoning effort, builtin_/system_ tool namespaces, the python
tool without a schema), developer message (instructions and the other tool namespaces), user
message."""
from __future__ import annotations

from typing import Optional

from .config import ConversationConfig
from .harmony import Conversation, Message, Role, developer_text, system_text
from .mcp_executor import ToolNamespaceConfig, is_system_namespace


def to_harmony_namespace(namespace: str) -> str:
    for prefix in ("builtin_", "system_"):
        if namespace.startswith(prefix):
            return namespace[len(prefix):]
    return namespace


class ConversationBuilder:
    def __init__(self, config: ConversationConfig):
        self.config = config

    def build(self, user_prompt: str,
              tool_configs: Optional[list[ToolNamespaceConfig]] = None) -> Conversation:
        sys_tools, dev_tools = {}, {}
        for tc in tool_configs or []:
            if is_system_namespace(tc.name):
                ns = to_harmony_namespace(tc.name)
                sys_tools[ns] = [] if ns == "python" else list(tc.tools)
            else:
                dev_tools[tc.name] = list(tc.tools)
        effort = self.config.reasoning_effort.lower()
        effort = effort if effort in ("low", "medium", "high") else "medium"
        msgs = [Message.from_role_and_content(Role.SYSTEM, system_text(
            self.config.model_identity, effort, self.config.conversation_start_date, sys_tools))]
        dev = developer_text(self.config.dev_instructions, dev_tools)
        if dev:
            msgs.append(Message.from_role_and_content(Role.DEVELOPER, dev))
        msgs.append(Message.from_role_and_content(Role.USER, user_prompt))
        return Conversation.from_messages(msgs)

    def append_user_message(self, conversation: Conversation, user_prompt: str) -> Conversation:
        return Conversation.from_messages(list(conversation.messages)
                                          + [Message.from_role_and_content(Role.USER, user_prompt)])
