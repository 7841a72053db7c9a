"""CPU oracle for the quantised-LLM hot path (TEST INFRASTRUCTURE, not product code).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs (``cpu_baseline`` and
``--impl reference``) may import this package, and only as the checker or the timed CPU baseline.
The product path (the ``q4b`` package and its CUDA library) never imports, links or calls it.

Parity of this restatement is pinned against golden vectors produced by importing the reference's
own ``scripts/llm/llama_q4.py`` (see ``tests/golden/make_golden.py``) and checked by
``tests/test_oracle_golden.py``.
"""
