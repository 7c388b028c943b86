// ltx25-threads.h -- fork-join over host threads for the library's host code
// (the adaLN chains, the RoPE tables).
#pragma once

#include <system_error>
#include <thread>
#include <vector>

namespace ltx25 {

// Runs part(k) for every k in [0, parts): part 0 on the calling thread, the
// others on new threads, and returns once all are done.  A thread the system
// will not create (std::system_error) leaves its part to the calling thread,
// so a host short of threads runs slower instead of terminating.
template <class Part>
void run_parts(int parts, const Part& part)
{
  std::vector<std::thread> pool;
  std::vector<int> left;
  if (parts > 1) {
    pool.reserve((size_t)parts - 1);
    left.reserve((size_t)parts - 1);
    for (int k = 1; k < parts; ++k) {
      try {
        pool.emplace_back(part, k);
      } catch (const std::system_error&) {
        left.push_back(k);
      }
    }
  }
  part(0);
  for (int k : left) part(k);
  for (std::thread& t : pool) t.join();
}

}  // namespace ltx25
