"""The library's per-thread kernel choices and process-wide switches, checked
on the host (setting them makes no CUDA call): accepted ranges, the error
message of a rejected value, and that a plan set on one host thread does not
reach another."""
import threading

import pytest

from vk_compute_b200._lib import lib


def last_error() -> str:
    return lib().vkc_last_error().decode()


@pytest.mark.parametrize("setter,getter,top", [
    ("vkc_set_gemv_plan", "vkc_get_gemv_plan", 4),
    ("vkc_set_attention_plan", "vkc_get_attention_plan", 5),
])
def test_plan_ranges(setter, getter, top):
    L = lib()
    try:
        for v in range(top + 1):
            assert getattr(L, setter)(v) == 0
            assert getattr(L, getter)() == v
        for bad in (-1, top + 1):
            assert getattr(L, setter)(bad) != 0
            assert str(bad) in last_error() and f"0 to {top}" in last_error()
            assert getattr(L, getter)() == top  # a rejected value changes nothing
    finally:
        getattr(L, setter)(0)


def test_plans_belong_to_the_calling_thread():
    L = lib()
    seen = {}

    def other():
        seen["gemv"] = L.vkc_get_gemv_plan()
        seen["attention"] = L.vkc_get_attention_plan()
        seen["int_dot"] = L.vkc_get_gemv_int_dot()

    try:
        assert L.vkc_set_gemv_plan(2) == 0
        assert L.vkc_set_attention_plan(3) == 0
        L.vkc_set_gemv_int_dot(0)
        t = threading.Thread(target=other)
        t.start()
        t.join()
        assert seen == {"gemv": 0, "attention": 0, "int_dot": 1}
        assert (L.vkc_get_gemv_plan(), L.vkc_get_attention_plan(), L.vkc_get_gemv_int_dot()) == (2, 3, 0)
    finally:
        L.vkc_set_gemv_plan(0)
        L.vkc_set_attention_plan(0)
        L.vkc_set_gemv_int_dot(1)


def test_switches_round_trip():
    L = lib()
    pdl, timing = L.vkc_get_pdl(), L.vkc_get_timing()
    try:
        for v in (1, 0):
            L.vkc_set_pdl(v)
            assert L.vkc_get_pdl() == v
            L.vkc_set_timing(v)
            assert L.vkc_get_timing() == v
        L.vkc_set_pdl(7)  # any non-zero value turns a switch on
        assert L.vkc_get_pdl() == 1
    finally:
        L.vkc_set_pdl(pdl)
        L.vkc_set_timing(timing)
