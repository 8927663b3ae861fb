"""A minimal stand-in for the parts of SGLang the monokernel plugin reads (SGLang is not
installed here): the monokernel registry and spec types (``srt/monokernels/spec.py``), the
runtime context (``srt/runtime_context.py``) and the forward context
(``srt/model_executor/forward_context.py``). Test infrastructure only; it mirrors the
interface the reference plugin consumes (``sgl_amd_mono/deepseek_v41/spec.py:959-1001``,
``test/unit/test_deepseek_v41_spec.py:41-51``), not SGLang's implementation."""
