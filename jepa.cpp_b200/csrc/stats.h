// Small host statistics shared by the planners' host code.
#pragma once

#include <cstdint>

namespace jb {

// Mean and population variance of n values, two passes in double (first the mean, then the squared
// deviations of each value from it, in index order).
template <class At>
inline void two_pass_moments(int64_t n, At at, double & mean, double & var) {
    double s = 0.0;
    for (int64_t i = 0; i < n; i++) s += (double) at(i);
    mean = s / (double) n;
    double q = 0.0;
    for (int64_t i = 0; i < n; i++) {
        const double d = (double) at(i) - mean;
        q += d * d;
    }
    var = q / (double) n;
}

}  // namespace jb
