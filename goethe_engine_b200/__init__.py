"""goethe_engine_b200: a B200-native decoder-forward library behind the goethe-engine C ABI (``abi/gc.h``)."""
