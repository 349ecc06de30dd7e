/* Test infrastructure: prints "same" when both layouts agree field for field. */
#include <stdio.h>
#include <stddef.h>
int ref_layout(size_t *o);
int our_layout(size_t *o);
int main(void) {
    size_t a[64], b[64];
    int na = ref_layout(a), nb = our_layout(b), i;
    if (na != nb) { printf("count %d %d\n", na, nb); return 1; }
    for (i = 0; i < na; i++)
        if (a[i] != b[i]) { printf("field %d: %zu %zu\n", i, a[i], b[i]); return 1; }
    printf("same %d\n", na);
    return 0;
}
