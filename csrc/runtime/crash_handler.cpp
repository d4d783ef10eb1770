// crash_handler.cpp - print a native backtrace when the process dies on a
// fatal signal inside the runtime (SIGSEGV / SIGBUS / SIGFPE / SIGILL).
//
// Opt-in: installed only when RAB_CRASH_HANDLER=1 is set when the extension
// loads (bench.py and the benchmark programs set it; a library import alone
// leaves the process's signal handlers untouched).  The handler saves the
// sigaction it replaces; on a fatal signal it prints the backtrace, puts the
// previous action back and re-raises, so Python's faulthandler or a host
// application's own handler still runs and the exit status is unchanged.
#include <execinfo.h>
#include <signal.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace rab {

namespace {

constexpr int kSignals[] = {SIGSEGV, SIGBUS, SIGFPE, SIGILL};
constexpr int kNumSignals = sizeof(kSignals) / sizeof(kSignals[0]);
struct sigaction g_previous[kNumSignals];
bool g_installed = false;

void on_fatal(int sig, siginfo_t* info, void*) {
  char head[160];
  const int n = snprintf(head, sizeof(head),
                         "\n[rab] fatal signal %d (%s) at address %p; native backtrace:\n", sig,
                         strsignal(sig), info ? info->si_addr : nullptr);
  if (n > 0) (void)!write(2, head, static_cast<size_t>(n));
  void* frames[64];
  const int depth = backtrace(frames, 64);
  backtrace_symbols_fd(frames, depth, 2);
  // hand the signal to whatever was installed before us (default action if nothing)
  bool restored = false;
  for (int i = 0; i < kNumSignals; ++i)
    if (kSignals[i] == sig) {
      sigaction(sig, &g_previous[i], nullptr);
      restored = true;
    }
  if (!restored) signal(sig, SIG_DFL);
  raise(sig);
}

}  // namespace

void install_crash_handler() {
  const char* on = std::getenv("RAB_CRASH_HANDLER");
  if (g_installed || on == nullptr || std::strcmp(on, "1") != 0) return;
  struct sigaction sa;
  std::memset(&sa, 0, sizeof(sa));
  sa.sa_sigaction = on_fatal;
  sa.sa_flags = SA_SIGINFO | SA_RESETHAND;
  sigemptyset(&sa.sa_mask);
  for (int i = 0; i < kNumSignals; ++i) sigaction(kSignals[i], &sa, &g_previous[i]);
  g_installed = true;
}

}  // namespace rab
