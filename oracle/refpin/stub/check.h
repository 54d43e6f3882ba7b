/* TEST INFRASTRUCTURE. A small stand-in for libcheck (the unit-test library the reference's tests
 * are written against, tests/BUILD; not vendored and not installed here). It provides the subset of
 * libcheck those tests use, with libcheck's names and meaning, so the test files compile unchanged:
 *
 *   START_TEST/END_TEST, ck_assert, ck_assert_msg, ck_assert_{int,uint}_{eq,ne}, ck_assert_float_le,
 *   ck_assert_ptr_nonnull, suite_create, tcase_create, suite_add_tcase, tcase_add_test,
 *   tcase_add_loop_test, tcase_add_unchecked_fixture, tcase_set_timeout, srunner_create,
 *   srunner_set_fork_status, srunner_run_all, srunner_ntests_failed, srunner_free.
 *
 * Runs are always in-process (CK_NOFORK): a failed assertion prints file:line and the message and
 * jumps out of the test case, which counts as one failure; the other cases still run. The summary
 * line has libcheck's form ("NN%: Checks: N, Failures: F, Errors: 0"). Timeouts are not enforced. */
#ifndef REFPIN_STUB_CHECK_H
#define REFPIN_STUB_CHECK_H
#include <setjmp.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

enum fork_status { CK_FORK_GETENV, CK_FORK, CK_NOFORK };
enum print_output { CK_SILENT, CK_MINIMAL, CK_NORMAL, CK_VERBOSE, CK_ENV, CK_SUBUNIT, CK_LAST };

typedef void (*ck_test_fn)(int);
typedef void (*ck_fixture_fn)(void);

#define CK_MAX_TESTS 64
#define CK_MAX_TCASES 16

typedef struct TCase
{
    const char *name;
    struct { const char *name; ck_test_fn fn; int start, end; } tests[CK_MAX_TESTS];
    int n_tests;
    ck_fixture_fn setup[4], teardown[4];
    int n_fixtures;
} TCase;

typedef struct Suite
{
    const char *name;
    TCase *tcases[CK_MAX_TCASES];
    int n_tcases;
} Suite;

typedef struct SRunner
{
    Suite *suite;
    int checks, failures;
} SRunner;

static jmp_buf ck_jump_out;

#define START_TEST(name) static void name(int _i __attribute__((unused)))
#define END_TEST

#define ck_fail_if_not_(cond, text, ...)                                                              \
    do                                                                                                \
    {                                                                                                 \
        if (!(cond))                                                                                  \
        {                                                                                             \
            fprintf(stderr, "%s:%d: Assertion '%s' failed: ", __FILE__, __LINE__, text);              \
            fprintf(stderr, __VA_ARGS__);                                                             \
            fputc('\n', stderr);                                                                      \
            longjmp(ck_jump_out, 1);                                                                  \
        }                                                                                             \
    } while (0)
#define ck_assert_msg(expr, ...) ck_fail_if_not_(expr, #expr, __VA_ARGS__)
#define ck_assert(expr) ck_fail_if_not_(expr, #expr, "%s", "")
#define ck_ck_cmp_(T, F, a, op, b)                                                                    \
    do                                                                                                \
    {                                                                                                 \
        T ck_a_ = (T)(a), ck_b_ = (T)(b);                                                             \
        ck_fail_if_not_(ck_a_ op ck_b_, #a " " #op " " #b, "(" F " vs " F ")", ck_a_, ck_b_);         \
    } while (0)
#define ck_assert_int_eq(a, b) ck_ck_cmp_(long long, "%lld", a, ==, b)
#define ck_assert_int_ne(a, b) ck_ck_cmp_(long long, "%lld", a, !=, b)
#define ck_assert_uint_eq(a, b) ck_ck_cmp_(unsigned long long, "%llu", a, ==, b)
#define ck_assert_uint_ne(a, b) ck_ck_cmp_(unsigned long long, "%llu", a, !=, b)
#define ck_assert_float_le(a, b) ck_ck_cmp_(double, "%g", a, <=, b)
#define ck_assert_ptr_nonnull(p) ck_assert_msg((p) != NULL, "%s is NULL", #p)

static inline __attribute__((unused)) Suite *suite_create(const char *name)
{
    Suite *s = (Suite *)calloc(1, sizeof(Suite));
    s->name = name;
    return s;
}

static inline __attribute__((unused)) TCase *tcase_create(const char *name)
{
    TCase *t = (TCase *)calloc(1, sizeof(TCase));
    t->name = name;
    return t;
}

static inline __attribute__((unused)) void suite_add_tcase(Suite *s, TCase *t)
{
    if (s->n_tcases < CK_MAX_TCASES)
        s->tcases[s->n_tcases++] = t;
}

static inline __attribute__((unused)) void ck_add_test_(TCase *t, const char *name, ck_test_fn fn, int start, int end)
{
    if (t->n_tests < CK_MAX_TESTS)
    {
        t->tests[t->n_tests].name = name;
        t->tests[t->n_tests].fn = fn;
        t->tests[t->n_tests].start = start;
        t->tests[t->n_tests].end = end;
        t->n_tests++;
    }
}
#define tcase_add_test(t, fn) ck_add_test_(t, #fn, fn, 0, 1)
#define tcase_add_loop_test(t, fn, s, e) ck_add_test_(t, #fn, fn, s, e)

static inline __attribute__((unused)) void tcase_add_unchecked_fixture(TCase *t, ck_fixture_fn setup,
                                                                        ck_fixture_fn teardown)
{
    if (t->n_fixtures < 4)
    {
        t->setup[t->n_fixtures] = setup;
        t->teardown[t->n_fixtures] = teardown;
        t->n_fixtures++;
    }
}

static inline __attribute__((unused)) void tcase_set_timeout(TCase *t, double seconds)
{
    (void)t;
    (void)seconds;
}

static inline __attribute__((unused)) SRunner *srunner_create(Suite *s)
{
    SRunner *r = (SRunner *)calloc(1, sizeof(SRunner));
    r->suite = s;
    return r;
}

static inline __attribute__((unused)) void srunner_set_fork_status(SRunner *r, enum fork_status f)
{
    (void)r;
    (void)f;
}

static inline __attribute__((unused)) void srunner_run_all(SRunner *r, enum print_output mode)
{
    Suite *s = r->suite;
    for (int c = 0; c < s->n_tcases; ++c)
    {
        TCase *t = s->tcases[c];
        for (int f = 0; f < t->n_fixtures; ++f)
            if (t->setup[f])
                t->setup[f]();
        for (int k = 0; k < t->n_tests; ++k)
        {
            for (int i = t->tests[k].start; i < t->tests[k].end; ++i)
            {
                r->checks++;
                if (setjmp(ck_jump_out) == 0)
                {
                    t->tests[k].fn(i);
                    if (mode == CK_VERBOSE)
                        fprintf(stderr, "%s:%s:%s:%d: Passed\n", s->name, t->name, t->tests[k].name, i);
                }
                else
                {
                    r->failures++;
                    fprintf(stderr, "%s:%s:%s:%d: Failed\n", s->name, t->name, t->tests[k].name, i);
                }
            }
        }
        for (int f = t->n_fixtures - 1; f >= 0; --f)
            if (t->teardown[f])
                t->teardown[f]();
    }
    if (mode != CK_SILENT)
        fprintf(stdout, "%d%%: Checks: %d, Failures: %d, Errors: 0\n",
                r->checks ? 100 * (r->checks - r->failures) / r->checks : 100, r->checks, r->failures);
}

static inline __attribute__((unused)) int srunner_ntests_failed(SRunner *r)
{
    return r->failures;
}

static inline __attribute__((unused)) void srunner_free(SRunner *r)
{
    Suite *s = r->suite;
    for (int c = 0; c < s->n_tcases; ++c)
        free(s->tcases[c]);
    free(s);
    free(r);
}

#endif
