from tileops.testing.test_base import (
    TestBase,
    allclose_compare,
    exact_compare,
    get_check_result,
    record_check_result,
)

__all__ = [
    "TestBase",
    "allclose_compare",
    "exact_compare",
    "get_check_result",
    "record_check_result",
]
