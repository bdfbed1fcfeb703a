"""Host-side logic that needs no GPU: the elementwise fusion-plan cache."""
import pytest


def test_plan_cache_counts_hits_per_chain():
    from torchcl.jit.cache import PlanCache
    built = []
    cache = PlanCache()

    def build(chain):
        built.append(chain)
        return ("plan", chain)

    a = cache.plan_for(("add", ("relu",)), build)
    b = cache.plan_for(("add", ("relu",)), build)
    c = cache.plan_for((None, ("sigmoid", "relu")), build)
    assert a is b and c != a
    assert built == [("add", ("relu",)), (None, ("sigmoid", "relu"))]
    assert cache.stats() == {"hits": 1, "misses": 2, "size": 2}
    cache.clear()
    assert len(cache) == 0 and cache.stats()["hits"] == 0


def test_plan_cache_keeps_nothing_when_a_build_fails():
    from torchcl.jit.cache import PlanCache
    cache = PlanCache()

    def build(chain):
        raise ValueError("Unknown unary op for fusion")

    with pytest.raises(ValueError):
        cache.plan_for(("add", ("nope",)), build)
    assert ("add", ("nope",)) not in cache and cache.stats()["misses"] == 0


def test_jit_plans_do_not_depend_on_the_element_count():
    """The reference keys its kernels by source text that embeds n; a plan here is the
    op-code list alone, so one chain is built once whatever the sizes."""
    from torchcl.jit import compiler
    from torchcl.jit.cache import get_kernel_cache
    jit = compiler.JITCompiler()
    cache = get_kernel_cache()
    before = cache.stats()
    p1 = jit._plan("mul", ["tanh", "neg"])
    p2 = jit._plan("mul", ["tanh", "neg"])
    assert p1 is p2 and p1[1] == 2 and list(p1[0]) == [3, 4]
    after = cache.stats()
    assert after["hits"] >= before["hits"] + 1
    with pytest.raises(ValueError):
        jit._plan(None, ["nope"])


def test_pool_free_from_a_finalizer_inside_a_locked_section():
    """A handle's finalizer may run (through a garbage collection) while this thread
    is inside one of the pool's locked sections; its free() must not wait for the
    lock its own thread holds."""
    import threading
    from torchcl.runtime.memory import CLBuffer, CLBufferPool
    pool = CLBufferPool()
    buf = CLBuffer(0, 64, 64)  # a NULL block: ojx_free(NULL) is a no-op
    done = threading.Event()

    def run():
        with pool._lock:  # as if a GC fired inside allocate()'s critical section
            pool.free(buf)
        done.set()

    t = threading.Thread(target=run, daemon=True)
    t.start()
    t.join(timeout=10)
    assert done.is_set(), "free() inside the pool's own locked section deadlocked"
    assert buf._freed
