"""Small helpers: `value_or` and a method LRU cache that does not keep `self` alive."""
import functools
import weakref
from typing import Any, Optional


def value_or(value: Optional[Any], default: Any) -> Any:
    """`value` unless it is None, else `default`."""
    return default if value is None else value


def weak_lru(maxsize: Optional[int] = 128, typed: bool = False):
    """`functools.lru_cache` for methods, keyed on a weak reference to the instance (a plain
    lru_cache on a method keeps every instance it has seen alive)."""
    def deco(func):
        @functools.lru_cache(maxsize, typed)
        def cached(self_ref, *args, **kwargs):
            return func(self_ref(), *args, **kwargs)

        @functools.wraps(func)
        def method(self, *args, **kwargs):
            return cached(weakref.ref(self), *args, **kwargs)
        return method
    return deco
