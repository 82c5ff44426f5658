"""Prefill / decode disaggregation: a prefill engine computes the prompt and the
first token, then hands the sequence's KV blocks to a decode engine.

* ``protocol``    framed JSON control messages ([u32 length][JSON]).
* ``kv_channel``  whole-block KV export / import: in-process, TCP with pinned
                  host staging, or NVLink (the prefill GPU writes straight into
                  the decode GPU's pool through a CUDA IPC mapping).
* ``serve``       the collocated / prefill / decode serving roles.
"""
