"""B200-native YOLOv8/YOLO11 inference engine (sm_100a).

The engine itself is native code (``csrc/`` -> ``lib/libyolob200.so`` and ``bin/yolocuda``)
behind the reference's ``yolo.h`` C ABI.  This Python package holds the host-side helpers
around it: the seeded random-init model zoo (``nn``), the model-directory writer
(``export``), the synthetic frame generator (``frames``), the build step (``build``), a
ctypes binding of the C ABI (``runtime``) and the gRPC batching server (``serve``).
"""
