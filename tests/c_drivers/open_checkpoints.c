/* Opens every checkpoint named on the command line, or every file of the one
 * directory named, with the library's parser and admission catalogue
 * (lun_weights_open in lunelette_b200/csrc/weights.c over csrc/st.c) and prints
 * one verdict line per file: "<rc> <error message>". Built with the address
 * and undefined-behaviour sanitizers by tests/test_host.py, so a memory error
 * on any input ends the run with the sanitizer's report. */
#include <dirent.h>
#include <stdio.h>
#include <string.h>
#include <sys/stat.h>

#include "weights.h"

static void open_one(const char *path)
{
    lun_weights w;
    char error[512] = "";
    int rc = lun_weights_open(&w, path, error, sizeof error);
    if (rc == 0) {
        lun_weights_close(&w);
    }
    printf("%d %s\n", rc, error);
}

int main(int argc, char **argv)
{
    struct stat st;
    if (argc == 2 && stat(argv[1], &st) == 0 && S_ISDIR(st.st_mode)) {
        DIR *dir = opendir(argv[1]);
        if (!dir) {
            return 2;
        }
        char path[4096];
        for (struct dirent *e = readdir(dir); e; e = readdir(dir)) {
            if (e->d_name[0] == '.') {
                continue;
            }
            snprintf(path, sizeof path, "%s/%s", argv[1], e->d_name);
            open_one(path);
        }
        closedir(dir);
        return 0;
    }
    for (int i = 1; i < argc; i++) {
        open_one(argv[i]);
    }
    return 0;
}
