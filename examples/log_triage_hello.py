"""One chat turn that triages a few log lines, with timing of load, engine build and the turn (the
reference's LogTriageHelloWorld, on this engine).

    python examples/log_triage_hello.py [MODEL]
"""
import sys
import time

import demo_models  # noqa: F401
from demo_models import chat_model

from nanovllm_b200.api.factory import LlmModelFactory
from nanovllm_b200.chat import LlmListeners
from nanovllm_b200.llm import LLM

PROMPT = """You are helping an on-call engineer. Read the log lines and reply in three short bullets:
1) what failed
2) likely cause
3) one concrete next check
Do not invent hosts or error codes that are not in the log.
Log:
2026-08-07 22:14:01 WARN  payment-api - retry 1/3 for order=99102 cause=SocketTimeoutException
2026-08-07 22:14:04 WARN  payment-api - retry 2/3 for order=99102 cause=SocketTimeoutException
2026-08-07 22:14:08 ERROR payment-api - give up order=99102 after 3 timeouts upstream=billing-svc:8443
2026-08-07 22:14:08 INFO  payment-api - marked order=99102 status=PAYMENT_FAILED"""


def _timing(what: str, t0: float) -> None:
    ms = (time.perf_counter() - t0) * 1000
    print(f"[timing] {what}: " + (f"{ms:.0f} ms" if ms < 1000 else f"{ms / 1000:.2f} s"))


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    path = chat_model(argv[0] if argv else None)
    t_all = t0 = time.perf_counter()
    model = LlmModelFactory.make(path)
    _timing("model load", t0)
    t0 = time.perf_counter()
    llm = LLM.builder(model).max_model_len(2048).max_num_seqs(2).system_prompt("") \
        .listen(LlmListeners.silent()).build()
    _timing("engine build", t0)
    t0 = time.perf_counter()
    advice = llm.chat(128).send(PROMPT).answer
    _timing("chat turn", t0)
    print("\n" + advice)
    _timing("total", t_all)
    llm.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
