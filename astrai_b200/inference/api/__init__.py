"""HTTP API: generation loop with stop sequences, OpenAI / Anthropic formats, tool parsing, FastAPI server."""

from astrai_b200.inference.api.anthropic import AnthropicResponseBuilder
from astrai_b200.inference.api.openai import OpenAIResponseBuilder
from astrai_b200.inference.api.protocol import (GenContext, ProtocolHandler, ResponseBuilder, StopChecker, StopInfo,
                                                sse_done, sse_event)
from astrai_b200.inference.api.server import (AnthropicMessage, ChatCompletionRequest, ChatMessage, FunctionDef,
                                              MessagesRequest, ToolDef, get_app, run_server)
from astrai_b200.inference.api.tool_parser import BaseToolParser, SimpleJsonToolParser, ToolParserFactory

__all__ = ["AnthropicMessage", "AnthropicResponseBuilder", "BaseToolParser", "ChatCompletionRequest", "ChatMessage",
           "FunctionDef", "GenContext", "MessagesRequest", "OpenAIResponseBuilder", "ProtocolHandler",
           "ResponseBuilder", "SimpleJsonToolParser", "StopChecker", "StopInfo", "ToolDef", "ToolParserFactory",
           "get_app", "run_server", "sse_done", "sse_event"]
