from kavor_b200.engine.llm_engine import LLMEngine


class LLM(LLMEngine):
    """Offline inference entry point (kavor/llm.py)."""
