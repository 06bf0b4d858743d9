"""The scheduler's page moves (fmd_scheduler.cu k_schedule). Thread 0 keeps
the bookkeeping serial: a finished slot's pages go onto the free stack at
[free_top, free_top + n) and an admitted slot's page k is stack entry
free_top - 1 - k. The copies themselves are recorded and done afterwards by
all threads, frees before admissions (a barrier between them). Restated here
in Python, the recorded-then-copied form gives the same page tables and free
stack as moving one page at a time in the serial loop, over random sequences
of finishes and admissions, including a slot freed and re-admitted in the
same step."""

from __future__ import annotations

import random

import pytest


def serial_step(stack, top, table, finished, admitted):
    for slot in finished:
        for p in table[slot]:
            stack[top] = p
            top += 1
        table[slot] = []
    for slot, need in admitted:
        pages = []
        for _ in range(need):
            top -= 1
            pages.append(stack[top])
        table[slot] = pages
    return top


def recorded_step(stack, top, table, finished, admitted):
    frees = []
    for slot in finished:  # thread 0: record, advance the top
        frees.append((slot, list(table[slot]), top))
        top += len(table[slot])
        table[slot] = []
    for slot, pages, base in frees:  # all threads: copy (any order)
        order = list(range(len(pages)))
        random.shuffle(order)
        for k in order:
            stack[base + k] = pages[k]
    allocs = []
    for slot, need in admitted:  # thread 0, after the barrier: record
        allocs.append((slot, need, top))
        top -= need
    for slot, need, t0 in allocs:  # all threads
        table[slot] = [None] * need
        order = list(range(need))
        random.shuffle(order)
        for k in order:
            table[slot][k] = stack[t0 - 1 - k]
    return top


@pytest.mark.parametrize("seed", range(30))
def test_recorded_page_moves_match_the_serial_moves(seed):
    rng = random.Random(seed)
    random.seed(seed + 1000)
    n_pages, slots = 400, 32
    a_stack, b_stack = list(range(n_pages)) + [None] * 8, list(range(n_pages)) + [None] * 8
    a_top = b_top = n_pages
    a_tab = {s: [] for s in range(slots)}
    b_tab = {s: [] for s in range(slots)}
    for _ in range(60):
        busy = [s for s in range(slots) if a_tab[s]]
        finished = rng.sample(busy, rng.randint(0, min(4, len(busy))))
        free_now = [s for s in range(slots) if not a_tab[s] or s in finished]
        admitted, top_after = [], a_top + sum(len(a_tab[s]) for s in finished)
        for s in rng.sample(free_now, rng.randint(0, min(4, len(free_now)))):
            need = rng.randint(1, 40)
            if need > top_after:
                break
            admitted.append((s, need))
            top_after -= need
        a_top = serial_step(a_stack, a_top, a_tab, finished, admitted)
        b_top = recorded_step(b_stack, b_top, b_tab, finished, admitted)
        assert a_top == b_top
        assert a_stack[:a_top] == b_stack[:b_top]
        assert a_tab == b_tab
    # every page is either on the stack or in exactly one table
    held = sorted(p for s in a_tab for p in a_tab[s])
    assert sorted(a_stack[:a_top] + held) == list(range(n_pages))
