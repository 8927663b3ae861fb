"""SGLang's logits processor output (a test stand-in)."""

from dataclasses import dataclass
from typing import Any


@dataclass
class LogitsProcessorOutput:
    next_token_logits: Any = None
    hidden_states: Any = None
