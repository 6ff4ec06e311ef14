// C-ABI plumbing shared by all entry points: the thread-local error message
// and the ABI version.
#include "common.cuh"

namespace unum {

static thread_local char g_err[512] = {0};

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

void clear_error() { g_err[0] = 0; }

}  // namespace unum

extern "C" const char *unum_last_error(void) { return unum::g_err; }

extern "C" int unum_abi_version(void) { return 102; }
