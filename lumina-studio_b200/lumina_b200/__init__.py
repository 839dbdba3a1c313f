"""B200-native Lumina decode path.

Hot path in ``liblumina_cuda.so`` (hand-written sm_100a CUDA, C ABI declared
in ``include/lumina_cuda.h``); this package is the host side that mirrors the
reference's Python interface for the path:

  * ``lumina_b200.cuda``    — ctypes boundary in the style of the reference's
    ``tops.py`` (version check, self-test, ``{"error"}`` convention)
  * ``lumina_b200.loader``  — ``.lumina`` records straight to device memory
  * ``lumina_b200.engine``  — ``CudaChatModel`` (the ChatModel drop-in) and the
    greedy drivers ``generate`` / ``generate_cached`` / tree verify
  * ``lumina_b200.synthetic`` — seeded workloads
"""
