// Host-only check of lf::PerContextOnce (csrc/lf_common.cuh): the set-up step runs once per
// context id, again for a context it has not seen, again after a failed attempt, and again for
// a context evicted past the table's 64 entries.  The context id comes from a stub here, so the
// program needs no GPU; it prints "ok" and exits 0 when every check holds.
#include "../../loopfuse_b200/csrc/lf_common.cuh"

#include <stdarg.h>

namespace lf {
static unsigned long long g_ctx = 1;
static bool g_ctx_fails = false;
int current_context_id(unsigned long long* id) {
    if (g_ctx_fails) return LF_ECUDA;
    *id = g_ctx;
    return LF_OK;
}
int set_error(int code, const char*, ...) { return code; }
void clear_error() {}
bool register_device_error_reader(DeviceErrorReader) { return true; }
}  // namespace lf

#define EXPECT(c)                                                  \
    do {                                                           \
        if (!(c)) {                                                \
            fprintf(stderr, "line %d: check failed: %s\n", __LINE__, #c); \
            return 1;                                              \
        }                                                          \
    } while (0)

int main() {
    lf::PerContextOnce once;
    int runs = 0, rc_step = LF_OK;
    auto step = [&] {
        ++runs;
        return rc_step;
    };
    lf::g_ctx = 1;
    EXPECT(once.run(step) == LF_OK && runs == 1);
    EXPECT(once.run(step) == LF_OK && runs == 1);          // same context: cached
    lf::g_ctx = 2;
    EXPECT(once.run(step) == LF_OK && runs == 2);          // another context: runs
    lf::g_ctx = 1;
    EXPECT(once.run(step) == LF_OK && runs == 2);
    lf::g_ctx = 3;
    rc_step = LF_ECUDA;
    EXPECT(once.run(step) == LF_ECUDA && runs == 3);       // failure is returned, not cached
    rc_step = LF_OK;
    EXPECT(once.run(step) == LF_OK && runs == 4);
    EXPECT(once.run(step) == LF_OK && runs == 4);
    lf::g_ctx_fails = true;
    EXPECT(once.run(step) == LF_ECUDA && runs == 4);       // no context id: no set-up
    lf::g_ctx_fails = false;
    for (unsigned long long c = 100; c < 100 + 64; ++c) {  // 64 new contexts evict 1, 2 and 3
        lf::g_ctx = c;
        EXPECT(once.run(step) == LF_OK);
    }
    EXPECT(runs == 4 + 64);
    lf::g_ctx = 163;
    EXPECT(once.run(step) == LF_OK && runs == 68);         // still held
    lf::g_ctx = 1;
    EXPECT(once.run(step) == LF_OK && runs == 69);         // evicted: runs again
    printf("ok\n");
    return 0;
}
