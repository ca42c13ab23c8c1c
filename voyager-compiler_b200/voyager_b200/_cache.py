"""A cache keyed by tensor identity.

``weakref.WeakKeyDictionary`` compares keys with ``==``, which a tensor
evaluates elementwise; this cache keys on ``id()`` and drops an entry when
its tensor is collected.
"""

import threading
import weakref


class TensorCache:
    def __init__(self):
        self._d = {}
        self._lock = threading.Lock()

    def get(self, t, key):
        with self._lock:
            e = self._d.get(id(t))
            if e is None or e[0]() is not t:
                return None
            return e[1].get(key)

    def put(self, t, key, value):
        i = id(t)
        with self._lock:
            e = self._d.get(i)
            if e is None or e[0]() is not t:
                ref = weakref.ref(t, lambda _r, i=i, d=self._d: d.pop(i, None))
                e = (ref, {})
                self._d[i] = e
            e[1][key] = value
        return value

    def clear(self):
        with self._lock:
            self._d.clear()
