/* ref_sample.c - exposes the reference's own token sampler for parity checks (test infrastructure).
 *
 * Compiled by oracle/Makefile with the reference's unmodified sources, read in place from the
 * reference tree: src/chat.c is included so that its static sample() (chat.c:36-69) and pcg32()
 * (chat.c:27-33) can be called. The library lands in oracle/_ref/ and is only used as a checker.
 */
#include "chat.c"

/* One draw: the sampler state {temp, top_p, top_k, rng} as chat.c keeps it; *rng is advanced. */
int ref_sample(const float *logits, int V, float temp, float top_p, int top_k, uint64_t *rng)
{
    Sampler sp;
    sp.temp = temp;
    sp.top_p = top_p;
    sp.top_k = top_k;
    sp.rng = *rng;
    const int t = sample(&sp, logits, V);
    *rng = sp.rng;
    return t;
}
