"""Cross-request batching with one engine-owning worker thread.

Same contract as the reference BatchEngine (laya_cuda/batching.py:17-157): bounded pending
queue, collection for up to max_wait_ms after the oldest request, whole requests packed into
batches under max_batch_size questions and max_batch_tokens packed tokens (16-token row spans),
per-request futures with metrics.  A failing request fails only its own future, a failing batch
only that batch's futures, and a fatal worker error fails every accepted request before the
worker releases the GPU.

Unlike the reference's worker, which runs one synchronous Runtime.predict per batch
(batching.py:122), this one pipelines through Runtime.submit / collect: batch i+1 is packed and
launched before batch i is collected and decoded, and requests that arrive while a batch runs
are tokenised before it is collected, and a burst of requests is tokenised batch by batch (a
batch's requests together, through the adapter's prepare_many, which spreads the tokenizer over
a few helper threads), so tokenisation, packing and decoding overlap the device.  Every engine
and adapter call is made on the worker thread.
"""
from concurrent.futures import Future
from copy import deepcopy
import math
from queue import Full
from threading import Condition, Thread, current_thread
import time

from .engine import Engine
from .runtime import span


class _Prediction(Future):
    metrics: dict


def _copy_json(value):
    t = type(value)
    if t is str or t is int or t is float or t is bool or value is None:
        return value
    if t is dict:
        return {key: _copy_json(item) for key, item in value.items()}
    if t is list:
        return [_copy_json(item) for item in value]
    return deepcopy(value)


def snapshot(value):
    """A copy of a submitted state or question mapping, so later changes by the caller do not
    reach the request (the reference deep-copies both).  Plain dicts, lists and scalars, what
    JSON-like requests hold, are copied directly (a few times faster than deepcopy); anything
    else, and structures too deep or cyclic for that, goes through deepcopy."""
    try:
        return _copy_json(value)
    except RecursionError:
        return deepcopy(value)


class BatchEngine:
    def __init__(self, model="laya", *, max_batch_size=16, max_batch_tokens=4096, max_pending=128, max_wait_ms=1,
                 **engine_options):
        for value in (max_batch_size, max_batch_tokens, max_pending):
            if type(value) is not int or value < 1:
                raise ValueError("Batch and queue limits must be positive integers")
        if not math.isfinite(max_wait_ms) or max_wait_ms < 0:
            raise ValueError("max_wait_ms must be finite and nonnegative")
        if engine_options.get("backend", "cuda") != "cuda":
            raise ValueError("BatchEngine supports backend='cuda' only; use Engine for official")
        self.max_batch_size, self.max_batch_tokens = max_batch_size, max_batch_tokens
        self.max_pending, self.wait = max_pending, max_wait_ms / 1000
        self._cv, self._queue, self._pending, self._closed = Condition(), [], 0, False
        ready = Future()
        self._thread = Thread(target=self._worker, args=(model, engine_options, ready), name="laya-batch", daemon=True)
        self._thread.start()
        ready.result()

    def submit(self, state, questions):
        """A Future of the answer dict, with per-request `metrics`; raises queue.Full at capacity."""
        started = time.perf_counter()
        with self._cv:
            if self._closed:
                raise RuntimeError("BatchEngine is closed")
            if self._pending >= self.max_pending:
                raise Full("BatchEngine pending request limit reached")
            future = _Prediction()
            future.metrics = {}
            self._queue.append((future, snapshot(state), snapshot(questions), started))
            self._pending += 1
            self._cv.notify()
        return future

    def close(self):
        """Rejects new submissions and drains accepted requests before the GPU is released."""
        with self._cv:
            self._closed = True
            self._cv.notify_all()
        if current_thread() is not self._thread:
            self._thread.join()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _finish(self, request, result=None, error=None):
        future = request[0]
        with self._cv:
            self._pending -= 1
        if future.cancelled():
            return
        if error is None:
            future.set_result(result)
        else:
            future.set_exception(error)

    def _collect(self, block):
        """Takes the queued requests.  block=True waits for work and then up to max_wait_ms after
        the oldest request (the batching window); returns None when closed and drained.
        block=False (a batch is on the device) takes only what is queued now, possibly []."""
        with self._cv:
            if block:
                self._cv.wait_for(lambda: self._queue or self._closed)
            if not self._queue:
                return None if self._closed else []
            if block:
                deadline = self._queue[0][3] + self.wait
                while not self._closed and len(self._queue) < self.max_batch_size:
                    remaining = deadline - time.perf_counter()
                    if remaining <= 0:
                        break
                    self._cv.wait(remaining)
            taken, self._queue = self._queue, []
            return taken

    def _prepare(self, engine, active, waiting, prepared):
        """Tokenises the next taken requests (already in `active`): those whose questions fit
        what is left of the question budget after `prepared` (at least one; a request has one
        item per question).  Returns their (request, items, packed tokens) entries; a request
        that was cancelled or failed is resolved and dropped.  Several requests go to the
        adapter's prepare_many when it has one (tokenised in parallel, on this thread's call)."""
        room = self.max_batch_size - sum(len(entry[1]) for entry in prepared)
        chunk = []
        while waiting:
            size = self._questions(waiting[0])
            if chunk and size > room:
                break
            request = waiting.pop(0)
            room -= size
            if request[0].set_running_or_notify_cancel():
                chunk.append(request)
            else:
                self._finish(request)
                active.remove(request)
        many = getattr(engine.adapter, "prepare_many", None)
        if many is not None and len(chunk) > 1:
            results = many([(request[1], request[2]) for request in chunk])
        else:
            results = []
            for request in chunk:
                try:
                    results.append(engine.adapter.prepare(request[1], request[2]))
                except Exception as error:
                    results.append(error)
        entries = []
        for request, items in zip(chunk, results):
            try:
                if isinstance(items, Exception):
                    raise items
                tokens = sum(span(len(item[0])) for item in items)
                if len(items) > self.max_batch_size or tokens > self.max_batch_tokens:
                    raise ValueError("Request exceeds batch budget; increase limits or submit fewer questions")
                entries.append((request, items, tokens))
            except Exception as error:
                active.remove(request)
                self._finish(request, error=error)
        return entries

    @staticmethod
    def _questions(request):
        """Items a taken request will have (one per question), known before tokenising."""
        questions = request[2]
        return len(questions) if isinstance(questions, dict) else 1

    def _fills(self, prepared, upcoming):
        """Whether the prepared requests reach one batch's question or token budget, or leave
        too little question room for the next waiting request, which then starts the next batch
        (first-fit would leave it out of this one anyway)."""
        questions = sum(len(entry[1]) for entry in prepared)
        return (questions >= self.max_batch_size
                or (prepared and questions + self._questions(upcoming) > self.max_batch_size)
                or sum(entry[2] for entry in prepared) >= self.max_batch_tokens)

    def _next_batch(self, prepared):
        """First-fit in arrival order under both budgets (questions and packed 16-token row spans);
        returns (batch, rest, questions)."""
        batch, rest, questions, tokens = [], [], 0, 0
        for entry in prepared:
            size = len(entry[1])
            if questions + size <= self.max_batch_size and tokens + entry[2] <= self.max_batch_tokens:
                batch.append(entry)
                questions += size
                tokens += entry[2]
            else:
                rest.append(entry)
        return batch, rest, questions

    def _fail(self, active, batch, error):
        for request, _, _ in batch:
            if request in active:
                active.remove(request)
                self._finish(request, error=error)

    def _launch(self, engine, active, batch, questions):
        """Packs and launches one batch without waiting for it; returns its in-flight record."""
        items = [item for _, rows, _ in batch for item in rows]
        executed = time.perf_counter()
        try:
            return batch, questions, executed, engine.runtime.submit(items)
        except Exception as error:
            self._fail(active, batch, error)
            return None

    def _complete(self, engine, active, batch, questions, executed, ticket):
        """Waits for a launched batch and resolves its requests' futures."""
        try:
            logits, acts, metrics = engine.runtime.collect(ticket)
        except Exception as error:
            self._fail(active, batch, error)
            return
        offset = 0
        for request, rows, _ in batch:
            future, _, questions_def, started = request
            try:
                end = offset + len(rows)
                result = engine.adapter.decode(logits[offset:end], acts[offset:end], questions_def, rows)
                future.metrics = {**metrics, "batch_questions": questions, "batch_requests": len(batch),
                                  "queue_ms": (executed - started) * 1000,
                                  "api_ms": (time.perf_counter() - started) * 1000,
                                  "tokens_per_question": [len(x[0]) for x in rows], "backend": "cuda",
                                  "precision": getattr(engine.runtime, "precision", "float16")}
                active.remove(request)
                self._finish(request, result)
            except Exception as error:
                if request in active:
                    active.remove(request)
                    self._finish(request, error=error)
            offset += len(rows)

    def _run(self, engine, active, taken, pending):
        """Tokenises and launches the taken requests batch by batch.  Requests are tokenised only
        as far as the next batch needs (by their question counts, then by the token budget), so
        a burst's later requests are tokenised while earlier batches run; each batch is launched
        before the previous one is collected and decoded (at most two batches in flight).
        Returns the last launched batch, still in flight, or None."""
        active.extend(taken)
        waiting, prepared = list(taken), []
        while waiting or prepared:
            while waiting and not self._fills(prepared, waiting[0]):
                prepared.extend(self._prepare(engine, active, waiting, prepared))
            if not prepared:
                break
            batch, prepared, questions = self._next_batch(prepared)
            launched = self._launch(engine, active, batch, questions)
            if pending is not None:
                self._complete(engine, active, *pending)
            pending = launched
        return pending

    def _worker(self, model, options, ready):
        engine, active, pending = None, [], None
        try:
            engine = Engine(model, **options)
            ready.set_result(None)
            while True:
                # With a batch in flight, requests queued meanwhile are tokenised before it is
                # collected; with none, wait for work and the batching window.
                taken = self._collect(block=pending is None)
                if taken is None:
                    break
                if not taken:
                    self._complete(engine, active, *pending)
                    pending = None
                    continue
                pending = self._run(engine, active, taken, pending)
            if pending is not None:
                self._complete(engine, active, *pending)
        except BaseException as error:
            with self._cv:
                self._closed = True
                active = (active or []) + self._queue
                self._queue = []
            if not ready.done():
                ready.set_exception(error)
            for request in active:
                if not request[0].running():
                    request[0].set_running_or_notify_cancel()
                self._finish(request, error=error)
        finally:
            if engine is not None:
                engine.close()
