"""BatchEngine contract with a fake engine (ports tests/test_batching.py of the reference):
one worker owns the engine, snapshots of inputs, packed budgets, cancellation, queue bounds,
per-request and per-batch failures, fatal-worker draining, close from a callback."""
from concurrent.futures import ThreadPoolExecutor, wait
from queue import Full
from threading import Event, get_ident
from types import SimpleNamespace

import pytest

from laya_cuda import BatchEngine
import laya_cuda.batching as batching


@pytest.fixture
def fake(monkeypatch):
    calls, owners = [], []
    entered, release = Event(), Event()
    release.set()

    class Engine:
        def __init__(self, *args, **kwargs):
            owners.append(get_ident())
            self.adapter = self
            self.runtime = self

        def prepare(self, state, questions):
            owners.append(get_ident())
            if not questions:
                raise ValueError("empty questions")
            return [([state] * definition, [0], 0) for definition in questions.values()]

        def predict(self, items):
            owners.append(get_ident())
            entered.set()
            assert release.wait(10)
            calls.append([len(x[0]) for x in items])
            if items[0][0][0] == "fatal":
                raise KeyboardInterrupt("worker stopped")
            if items[0][0][0] == "fail":
                raise RuntimeError("device failure")
            return [x[0][0] for x in items], [0] * len(items), {"gpu_ms": 1}

        # The worker launches a batch (submit) before collecting the previous one; the fake runs
        # the pass at submit and hands the result back at collect.
        def submit(self, items):
            self.tickets = getattr(self, "tickets", {})
            self.issued = ticket = getattr(self, "issued", 0) + 1
            self.tickets[ticket] = self.predict(items)
            return ticket

        def collect(self, ticket):
            return self.tickets.pop(ticket)

        def decode(self, logits, acts, questions, items):
            return dict(zip(questions, logits))

        def close(self):
            owners.append(get_ident())

    monkeypatch.setattr(batching, "Engine", Engine)
    return SimpleNamespace(calls=calls, owners=owners, entered=entered, release=release)


def test_merge_restore_snapshot_and_owner(fake):
    with BatchEngine(max_wait_ms=30) as engine:
        questions = {"same": 20, "second": 22}
        a = engine.submit("a", questions)
        questions.clear()
        b = engine.submit("b", {"same": 21})
        assert a.result(5) == {"same": "a", "second": "a"}
        assert b.result(5) == {"same": "b"}
        assert a.metrics["batch_requests"] == 2
        assert a.metrics["api_ms"] >= a.metrics["queue_ms"]
    assert fake.calls == [[20, 22, 21]]
    assert len(set(fake.owners)) == 1 and fake.owners[0] != get_ident()


def test_bounds_cancel_error_and_close(fake):
    fake.release.clear()
    engine = BatchEngine(max_pending=2, max_wait_ms=0)
    first = engine.submit("first", {"q": 20})
    assert fake.entered.wait(5)
    second = engine.submit("cancel", {"q": 20})
    assert second.cancel()
    with pytest.raises(Full):
        engine.submit("full", {"q": 20})
    fake.release.set()
    engine.close()
    assert first.result() == {"q": "first"} and second.cancelled()
    assert engine._pending == 0
    engine.close()
    with pytest.raises(RuntimeError, match="closed"):
        engine.submit("closed", {"q": 20})


def test_packed_budget_and_request_failure(fake):
    with BatchEngine(max_batch_size=4, max_batch_tokens=512, max_wait_ms=30) as engine:
        futures = [engine.submit(str(i), {"q": length}) for i, length in enumerate([20, 129, 24, 128])]
        assert [f.result(5) for f in futures] == [{"q": str(i)} for i in range(4)]
        for questions in ({}, dict.fromkeys(range(5), 20), {"q": 513}):
            with pytest.raises(ValueError):
                engine.submit("bad", questions).result(5)
        with pytest.raises(RuntimeError, match="device failure"):
            engine.submit("fail", {"q": 20}).result(5)
        assert engine.submit("ok", {"q": 20}).result(5) == {"q": "ok"}
    # Packed rows need no common length: one batch within 4 questions and 512 tokens.
    assert fake.calls[0] == [20, 129, 24, 128]
    assert engine._pending == 0


def test_concurrent_producers_and_callback_close(fake):
    with BatchEngine(max_wait_ms=2) as engine:
        with ThreadPoolExecutor(8) as pool:
            futures = list(pool.map(lambda i: engine.submit(str(i), {"q": 20}), range(64)))
        assert [f.result(5) for f in futures] == [{"q": str(i)} for i in range(64)]
        called = Event()

        def finish(future):
            engine.close()
            called.set()
        engine.submit("last", {"q": 20}).add_done_callback(finish)
        assert called.wait(5)


def test_initialization_failure(fake, monkeypatch):
    def fail(*args, **kwargs):
        raise FileNotFoundError("missing checkpoint")
    monkeypatch.setattr(batching, "Engine", fail)
    with pytest.raises(FileNotFoundError):
        BatchEngine()
    for options in ({"max_wait_ms": float("nan")}, {"max_pending": 0}, {"backend": "official"}):
        with pytest.raises(ValueError):
            BatchEngine(**options)


def test_fatal_worker_drains_and_notifies_cancelled_waiters(fake):
    fake.release.clear()
    engine = BatchEngine(max_wait_ms=0)
    failed = engine.submit("fatal", {"q": 20})
    assert fake.entered.wait(5)
    cancelled = engine.submit("cancel", {"q": 20})
    queued = engine.submit("queued", {"q": 20})
    assert cancelled.cancel()
    fake.release.set()
    done, pending = wait([failed, cancelled, queued], timeout=5)
    assert not pending and len(done) == 3
    for f in (failed, queued):
        with pytest.raises(KeyboardInterrupt):
            f.result()
    engine.close()
    assert engine._pending == 0


def test_split_results_follow_batch_order(fake):
    """Each request decodes its own slice of the batch's logits."""
    with BatchEngine(max_batch_size=8, max_wait_ms=30) as engine:
        futures = [engine.submit(s, {"x": n, "y": n + 1}) for s, n in (("p", 10), ("q", 30), ("r", 50))]
        assert [f.result(5) for f in futures] == [{"x": s, "y": s} for s in "pqr"]
        assert all(f.metrics["batch_questions"] == 6 for f in futures)


def test_next_batch_launches_before_the_previous_is_collected(monkeypatch):
    """Pipelining: with one question per batch, batch i+1 is submitted before batch i is
    collected and decoded, and no more than two batches are ever in flight."""
    events = []

    class Engine:
        def __init__(self, *args, **kwargs):
            self.adapter = self
            self.runtime = self
            self.inflight = 0

        def prepare(self, state, questions):
            return [([state], [0], 0) for _ in questions]

        def submit(self, items):
            self.inflight += 1
            assert self.inflight <= 2
            events.append(("submit", items[0][0][0]))
            return items[0][0][0]

        def collect(self, ticket):
            self.inflight -= 1
            events.append(("collect", ticket))
            return [ticket], [0], {"gpu_ms": 1}

        def decode(self, logits, acts, questions, items):
            events.append(("decode", logits[0]))
            return dict(zip(questions, logits))

        def close(self):
            pass

    monkeypatch.setattr(batching, "Engine", Engine)
    with BatchEngine(max_batch_size=1, max_wait_ms=50) as engine:
        futures = [engine.submit(s, {"q": 1}) for s in "abc"]
        assert [f.result(5) for f in futures] == [{"q": s} for s in "abc"]
    order = [e for e in events if e[0] != "decode"]
    assert order == [("submit", "a"), ("submit", "b"), ("collect", "a"), ("submit", "c"), ("collect", "b"),
                     ("collect", "c")]
    assert events.index(("decode", "a")) > events.index(("submit", "b"))


def test_burst_is_tokenised_batch_by_batch(monkeypatch):
    """A burst taken in one collection is not tokenised up front: the requests of batch i+1 are
    prepared after batch i has been launched, so tokenisation overlaps the device, and batches
    still keep arrival order within both budgets."""
    events = []

    class Engine:
        def __init__(self, *args, **kwargs):
            self.adapter = self
            self.runtime = self

        def prepare(self, state, questions):
            events.append(("prepare", state))
            return [([state] * 20, [0], 0) for _ in questions]

        def submit(self, items):
            events.append(("submit", tuple(item[0][0] for item in items)))
            return tuple(item[0][0] for item in items)

        def collect(self, ticket):
            return list(ticket), [0] * len(ticket), {"gpu_ms": 1}

        def decode(self, logits, acts, questions, items):
            return dict(zip(questions, logits))

        def close(self):
            pass

    monkeypatch.setattr(batching, "Engine", Engine)
    with BatchEngine(max_batch_size=2, max_wait_ms=50) as engine:
        futures = [engine.submit(s, {"q": 1}) for s in "abcde"]
        assert [f.result(5) for f in futures] == [{"q": s} for s in "abcde"]
    submits = [e[1] for e in events if e[0] == "submit"]
    assert submits == [("a", "b"), ("c", "d"), ("e",)]
    # Requests c and d are tokenised only after batch (a, b) was launched, e after (c, d).
    assert events.index(("prepare", "c")) > events.index(("submit", ("a", "b")))
    assert events.index(("prepare", "e")) > events.index(("submit", ("c", "d")))


def test_burst_is_prepared_in_chunks_on_the_worker(monkeypatch):
    """With an adapter that has prepare_many, a burst's requests are handed over in chunks that
    fill the next batch's question budget (counted before tokenising), on the worker thread; a
    request that fails in the chunk fails alone, and a chunk of one goes through prepare."""
    events, owners = [], set()

    class Engine:
        def __init__(self, *args, **kwargs):
            self.adapter = self
            self.runtime = self

        def prepare(self, state, questions):
            owners.add(get_ident())
            events.append(("prepare", state))
            return [([state] * 20, [0], 0) for _ in questions]

        def prepare_many(self, requests):
            owners.add(get_ident())
            events.append(("many", tuple(state for state, _ in requests)))
            return [ValueError(f"bad {state}") if state == "c" else self.prepare(state, questions)
                    for state, questions in requests]

        def submit(self, items):
            owners.add(get_ident())
            events.append(("submit", tuple(item[0][0] for item in items)))
            return tuple(item[0][0] for item in items)

        def collect(self, ticket):
            return list(ticket), [0] * len(ticket), {"gpu_ms": 1}

        def decode(self, logits, acts, questions, items):
            return dict(zip(questions, logits))

        def close(self):
            pass

    monkeypatch.setattr(batching, "Engine", Engine)
    with BatchEngine(max_batch_size=4, max_wait_ms=50) as engine:
        sizes = {"a": 1, "b": 2, "c": 1, "d": 1, "e": 3, "f": 2}
        futures = {s: engine.submit(s, {f"q{i}": 1 for i in range(n)}) for s, n in sizes.items()}
        for s, future in futures.items():
            if s == "c":
                with pytest.raises(ValueError, match="bad c"):
                    future.result(5)
            else:
                assert future.result(5) == {f"q{i}": s for i in range(sizes[s])}
    assert len(owners) == 1 and get_ident() not in owners
    # a + b + c fill the 4-question budget and go together; after c fails, d alone fills the
    # room left (one request: prepare); e (3) and f (2) do not fit one batch.
    assert [e[1] for e in events if e[0] == "many"] == [("a", "b", "c")]
    assert [tuple(dict.fromkeys(e[1])) for e in events if e[0] == "submit"] == [("a", "b", "d"), ("e",), ("f",)]


def test_snapshot_copies_like_deepcopy():
    """submit's snapshot: equal values and no shared mutable part for JSON-like requests (nested
    dicts and lists of scalars); other types and cycles go through deepcopy, so every input is
    copied as the reference's deepcopy copies it, and nesting too deep for deepcopy fails the
    same way."""
    from collections import OrderedDict
    from copy import deepcopy
    from laya_cuda.batching import snapshot
    questions = {"q": {"type": "choice", "instructions": {"ask": ["a", 1, 2.5, None, True]}, "criteria": ["x", "y"]}}
    copy = snapshot(questions)
    assert copy == deepcopy(questions)
    questions["q"]["criteria"].append("z")
    questions["q"]["instructions"]["ask"].clear()
    assert copy["q"]["criteria"] == ["x", "y"] and copy["q"]["instructions"]["ask"] == ["a", 1, 2.5, None, True]
    ordered = OrderedDict(a=[1])
    assert type(snapshot(ordered)) is OrderedDict and snapshot(ordered)["a"] is not ordered["a"]
    pair = ([1], "s")
    assert snapshot(pair) == pair and snapshot(pair)[0] is not pair[0]
    cyclic = {"a": []}
    cyclic["a"].append(cyclic)
    copied = snapshot(cyclic)
    assert copied["a"][0] is copied and copied is not cyclic
    def nested(depth):
        outer = value = []
        for _ in range(depth):
            value.append([])
            value = value[0]
        return outer
    assert snapshot(nested(300)) == nested(300)
    too_deep = nested(5000)
    with pytest.raises(RecursionError):
        deepcopy(too_deep)
    with pytest.raises(RecursionError):
        snapshot(too_deep)


def test_request_that_cannot_fit_starts_the_next_chunk(monkeypatch):
    """A waiting request whose questions exceed the room the prepared ones leave is not
    tokenised alone: the batch launches, and that request opens the next chunk."""
    events = []

    class Engine:
        def __init__(self, *args, **kwargs):
            self.adapter = self
            self.runtime = self

        def prepare(self, state, questions):
            events.append(("prepare", state))
            return [([state] * 20, [0], 0) for _ in questions]

        def prepare_many(self, requests):
            events.append(("many", tuple(state for state, _ in requests)))
            return [[([state] * 20, [0], 0) for _ in questions] for state, questions in requests]

        def submit(self, items):
            events.append(("submit", tuple(dict.fromkeys(item[0][0] for item in items))))
            return tuple(item[0][0] for item in items)

        def collect(self, ticket):
            return list(ticket), [0] * len(ticket), {"gpu_ms": 1}

        def decode(self, logits, acts, questions, items):
            return dict(zip(questions, logits))

        def close(self):
            pass

    monkeypatch.setattr(batching, "Engine", Engine)
    with BatchEngine(max_batch_size=4, max_wait_ms=50) as engine:
        sizes = {"a": 1, "b": 2, "c": 2, "d": 1}
        futures = [engine.submit(s, {f"q{i}": 1 for i in range(n)}) for s, n in sizes.items()]
        for future in futures:
            future.result(5)
    assert events == [("many", ("a", "b")), ("submit", ("a", "b")), ("many", ("c", "d")), ("submit", ("c", "d"))]
